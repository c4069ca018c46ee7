"""ctypes wrapper over the CPU oracle (oracle/kv_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU legs of bench.py, never by the product package.  See kv_oracle.h for what
is restated from the reference (src/model.cpp:1382-1445, 821-885, 1002-1059)
and for the assumptions A1-A6 (parity unpinned: ggml is not vendored).
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(HERE, "lib", "libkv_oracle.so")
_REF_PATH = os.path.join(HERE, "_ref", "libmoe_scalar.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)


class KvoCfg(ctypes.Structure):
    _fields_ = [
        ("n_head", ctypes.c_int32),
        ("n_head_kv", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("n_rot", ctypes.c_int32),
        ("rope_mode", ctypes.c_int32),
        ("n_ctx_orig", ctypes.c_int32),
        ("rope_base", ctypes.c_float),
        ("rope_freq_scale", ctypes.c_float),
        ("rope_attn_factor", ctypes.c_float),
        ("rope_ext_factor", ctypes.c_float),
        ("rope_beta_fast", ctypes.c_float),
        ("rope_beta_slow", ctypes.c_float),
        ("rope_freq_factors", _f32p),
        ("qk_norm", ctypes.c_int32),
        ("rms_eps", ctypes.c_float),
    ]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            import importlib.util
            spec = importlib.util.spec_from_file_location("_oracle_build", os.path.join(HERE, "build.py"))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            mod.build_oracle()
        L = ctypes.CDLL(_LIB_PATH)
        L.kvo_f32_to_f16.restype = ctypes.c_uint16
        L.kvo_f32_to_f16.argtypes = [ctypes.c_float]
        L.kvo_f16_to_f32.restype = ctypes.c_float
        L.kvo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.kvo_f32_to_f16_n.argtypes = [_f32p, _u16p, ctypes.c_int64]
        L.kvo_rope_corr_dims.argtypes = [ctypes.POINTER(KvoCfg), _f32p]
        L.kvo_rope_table.argtypes = [ctypes.POINTER(KvoCfg), ctypes.c_int64, ctypes.c_int64, _f32p]
        L.kvo_rms_norm_mul.argtypes = [_f32p, _f32p, ctypes.c_int32, ctypes.c_float, _f32p]
        L.kvo_rope_row.argtypes = [ctypes.POINTER(KvoCfg), _f32p, _f32p, _f32p]
        L.kvo_append.restype = ctypes.c_int
        L.kvo_append.argtypes = [ctypes.POINTER(KvoCfg), ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                 _f32p, ctypes.c_int64, _f32p, ctypes.c_int64, _f32p, ctypes.c_int64,
                                 _f32p, _f32p, _u16p, _u16p, _f32p]
        L.kvo_attend.restype = ctypes.c_int
        L.kvo_attend.argtypes = [ctypes.POINTER(KvoCfg), ctypes.c_int64, ctypes.c_int32,
                                 _f32p, _u16p, _u16p, _f32p, ctypes.c_int32]
        L.kvo_append_ring.restype = ctypes.c_int
        L.kvo_append_ring.argtypes = [ctypes.POINTER(KvoCfg), ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                      _f32p, ctypes.c_int64, _f32p, ctypes.c_int64, _f32p, ctypes.c_int64,
                                      _f32p, _f32p, _u16p, _u16p, _f32p]
        L.kvo_ngpt_norm.restype = None
        L.kvo_ngpt_norm.argtypes = [_f32p, _f32p, ctypes.c_int32, ctypes.c_float, _f32p]
        L.kvo_ring_mask.restype = None
        L.kvo_ring_mask.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, _f32p]
        L.kvo_attend_ex.restype = ctypes.c_int
        L.kvo_attend_ex.argtypes = [ctypes.POINTER(KvoCfg), ctypes.c_int64, ctypes.c_int32, _f32p, _u16p, _u16p,
                                    ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, _f32p,
                                    ctypes.c_int32]
        L.kvo_kv_cache_bytes.restype = ctypes.c_uint64
        L.kvo_kv_cache_bytes.argtypes = [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64]
        L.kvo_auto_n_ctx.restype = ctypes.c_int64
        L.kvo_auto_n_ctx.argtypes = [ctypes.c_int64, ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64]
        L.kvo_bits.restype = ctypes.c_uint64
        L.kvo_bits.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64]
        L.kvo_normal.restype = ctypes.c_float
        L.kvo_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64]
        L.kvo_gen_normal_f32.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, _f32p]
        L.kvo_gen_normal_f16.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, _u16p]
        L.kvo_gen_uniform_f32.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64,
                                          ctypes.c_float, ctypes.c_float, _f32p]
        L.kvo_gen_cache_rows.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _u16p]
        L.kvo_online_cores.restype = ctypes.c_int32
        _lib = L
    return _lib


def _p(a, t=_f32p):
    return None if a is None else a.ctypes.data_as(t)


class Oracle:
    """One layer's attention parameters plus the oracle entry points.

    `spec` is a kv_b200 model spec dict (n_head, n_head_kv, head_dim, n_rot,
    rope_mode, rope_base, ...).  The freq-factor array is kept alive here.
    """

    def __init__(self, spec):
        self.spec = dict(spec)
        ff = spec.get("rope_freq_factors")
        self._ff = None if ff is None else np.ascontiguousarray(ff, dtype=np.float32)
        c = KvoCfg()
        c.n_head = spec["n_head"]
        c.n_head_kv = spec["n_head_kv"]
        c.head_dim = spec["head_dim"]
        c.n_rot = spec.get("n_rot", spec["head_dim"])
        c.rope_mode = spec.get("rope_mode", 2)
        c.n_ctx_orig = spec.get("n_ctx_orig", 0)
        c.rope_base = spec.get("rope_base", 10000.0)
        c.rope_freq_scale = spec.get("rope_freq_scale", 1.0)
        c.rope_attn_factor = spec.get("rope_attn_factor", 1.0)
        c.rope_ext_factor = spec.get("rope_ext_factor", 0.0)
        c.rope_beta_fast = spec.get("rope_beta_fast", 0.0)
        c.rope_beta_slow = spec.get("rope_beta_slow", 0.0)
        c.rope_freq_factors = _p(self._ff)
        c.qk_norm = int(spec.get("qk_norm") or 0)   # True -> 1 (RMSNorm); 2 = nGPT
        c.rms_eps = spec.get("rms_eps", 1e-6)
        self.cfg = c

    # -- pieces ---------------------------------------------------------
    def rope_table(self, pos0, npos):
        half = self.cfg.n_rot // 2
        out = np.zeros((npos, half, 2), np.float32)
        lib().kvo_rope_table(ctypes.byref(self.cfg), pos0, npos, _p(out))
        return out

    def corr_dims(self):
        out = np.zeros(2, np.float32)
        lib().kvo_rope_corr_dims(ctypes.byref(self.cfg), _p(out))
        return out

    def rope_row(self, cs_row, x):
        x = np.ascontiguousarray(x, np.float32)
        cs_row = np.ascontiguousarray(cs_row, np.float32)
        y = np.empty_like(x)
        lib().kvo_rope_row(ctypes.byref(self.cfg), _p(cs_row), _p(x), _p(y))
        return y

    # -- the path ------------------------------------------------------
    def append(self, kcache, vcache, n_past, q, k, v, q_norm_w=None, k_norm_w=None):
        """q: [n_new, >=n_head*d] rows; k, v: [n_new, >=n_head_kv*d] rows (row
        strides taken from the arrays).  kcache/vcache: uint16 [n_ctx, hkv, d],
        modified in place.  Returns the rotated Q as [n_new, n_head, d] F32."""
        n_new = q.shape[0]
        for a in (q, k, v):
            assert a.dtype == np.float32 and a.strides[1] == 4
        assert kcache.flags.c_contiguous and vcache.flags.c_contiguous
        d, hq = self.cfg.head_dim, self.cfg.n_head
        q_out = np.zeros((n_new, hq, d), np.float32)
        qn = None if q_norm_w is None else np.ascontiguousarray(q_norm_w, np.float32)
        kn = None if k_norm_w is None else np.ascontiguousarray(k_norm_w, np.float32)
        rc = lib().kvo_append(ctypes.byref(self.cfg), kcache.shape[0], n_past, n_new,
                              _p(q), q.strides[0] // 4, _p(k), k.strides[0] // 4, _p(v), v.strides[0] // 4,
                              _p(qn), _p(kn), _p(kcache, _u16p), _p(vcache, _u16p), _p(q_out))
        assert rc == 0, rc
        return q_out

    def append_ring(self, kcache, vcache, pos0, q, k, v, q_norm_w=None, k_norm_w=None):
        """append() into a ring cache: kcache/vcache are uint16 [n_cells, hkv, d];
        the token at position p goes to cell p % n_cells (dory.c:459-522)."""
        n_new = q.shape[0]
        for a in (q, k, v):
            assert a.dtype == np.float32 and a.strides[1] == 4
        assert kcache.flags.c_contiguous and vcache.flags.c_contiguous
        d, hq = self.cfg.head_dim, self.cfg.n_head
        q_out = np.zeros((n_new, hq, d), np.float32)
        qn = None if q_norm_w is None else np.ascontiguousarray(q_norm_w, np.float32)
        kn = None if k_norm_w is None else np.ascontiguousarray(k_norm_w, np.float32)
        rc = lib().kvo_append_ring(ctypes.byref(self.cfg), kcache.shape[0], pos0, n_new,
                                   _p(q), q.strides[0] // 4, _p(k), k.strides[0] // 4, _p(v), v.strides[0] // 4,
                                   _p(qn), _p(kn), _p(kcache, _u16p), _p(vcache, _u16p), _p(q_out))
        assert rc == 0, rc
        return q_out

    def attend_ring(self, kcache, vcache, pos0, q_roped, mask=None, flash=False, n_threads=0):
        """Attention over a ring cache's cells in use (min(n_cells, pos0 + n_new))
        with dory's visibility mask (ring_mask), or the caller's mask over them."""
        n_new = q_roped.shape[0]
        n_cells = kcache.shape[0]
        n_used = min(n_cells, pos0 + n_new)
        if mask is None:
            mask = np.ascontiguousarray(ring_mask(n_cells, pos0, n_new)[:, :n_used])
        return self.attend_ex(kcache, vcache, n_used - n_new, q_roped, mask=mask, flash=flash,
                              n_threads=n_threads)

    def attend(self, kcache, vcache, n_past, q_roped, n_threads=0):
        q_roped = np.ascontiguousarray(q_roped, np.float32)
        n_new = q_roped.shape[0]
        out = np.zeros((n_new, self.cfg.n_head * self.cfg.head_dim), np.float32)
        rc = lib().kvo_attend(ctypes.byref(self.cfg), n_past, n_new, _p(q_roped),
                              _p(kcache, _u16p), _p(vcache, _u16p), _p(out), n_threads)
        assert rc == 0, rc
        return out


    def attend_ex(self, kcache, vcache, n_past, q_roped, mask=None, flash=False, n_threads=0):
        """attend() with the caller's additive mask (a float32 or float16 array of
        n_new rows of >= n_past+n_new keys; None = causal) and the flash-attn
        branch (kv_oracle.h A5, A6)."""
        q_roped = np.ascontiguousarray(q_roped, np.float32)
        n_new = q_roped.shape[0]
        out = np.zeros((n_new, self.cfg.n_head * self.cfg.head_dim), np.float32)
        mptr, mf16, mstride = None, 0, 0
        if mask is not None:
            mask = np.ascontiguousarray(mask)
            assert mask.dtype in (np.float32, np.float16) and mask.shape[0] == n_new
            mptr, mf16, mstride = mask.ctypes.data, int(mask.dtype == np.float16), mask.shape[1]
        rc = lib().kvo_attend_ex(ctypes.byref(self.cfg), n_past, n_new, _p(q_roped), _p(kcache, _u16p),
                                 _p(vcache, _u16p), mptr, mf16, mstride, int(bool(flash)), _p(out), n_threads)
        assert rc == 0, rc
        return out


# -- generators and helpers --------------------------------------------------

def ring_mask(n_cells, pos0, n_tokens):
    """dory_fill_attn_mask (dory.c:553-575) as F32 [n_tokens][n_cells] 0 / -inf."""
    out = np.empty((n_tokens, n_cells), np.float32)
    lib().kvo_ring_mask(n_cells, pos0, n_tokens, _p(out))
    return out


def f32_to_f16_bits(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().kvo_f32_to_f16_n(_p(x), _p(out, _u16p), x.size)
    return out


def gen_normal_f32(seed, stream, n, idx0=0):
    out = np.empty(n, np.float32)
    lib().kvo_gen_normal_f32(seed, stream, idx0, n, _p(out))
    return out


def gen_normal_f16(seed, stream, n, idx0=0):
    out = np.empty(n, np.uint16)
    lib().kvo_gen_normal_f16(seed, stream, idx0, n, _p(out, _u16p))
    return out


def gen_uniform_f32(seed, stream, n, lo, hi, idx0=0):
    out = np.empty(n, np.float32)
    lib().kvo_gen_uniform_f32(seed, stream, idx0, n, lo, hi, _p(out))
    return out


def gen_cache_rows(seed, stream, row0, nrows, n_head_kv, head_dim, h0=0, nh=None):
    nh = n_head_kv if nh is None else nh
    out = np.empty((nrows, nh, head_dim), np.uint16)
    lib().kvo_gen_cache_rows(seed, stream, row0, nrows, n_head_kv, head_dim, h0, nh, _p(out, _u16p))
    return out


def kv_cache_bytes(n_layer, n_head_kv, head_dim, n_ctx):
    return int(lib().kvo_kv_cache_bytes(n_layer, n_head_kv, head_dim, n_ctx))


def auto_n_ctx(avail, per_tok, n_ctx_train=0, longrope_orig=0):
    return int(lib().kvo_auto_n_ctx(avail, per_tok, n_ctx_train, longrope_orig))


def online_cores():
    return int(lib().kvo_online_cores())


# -- the reference's own scalar backend (oracle/_ref, built from its sources) -

class _RefBackend(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p),
        ("self", ctypes.c_void_p),
        ("matmul", ctypes.c_void_p),
        ("matmul_batch", ctypes.c_void_p),
        ("rmsnorm", ctypes.CFUNCTYPE(None, ctypes.c_void_p, _f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_float)),
        ("rope", ctypes.CFUNCTYPE(None, ctypes.c_void_p, _f32p, ctypes.c_int, _f32p, _f32p)),
        ("softmax", ctypes.CFUNCTYPE(None, ctypes.c_void_p, _f32p, ctypes.c_int)),
        ("swiglu", ctypes.c_void_p),
        ("begin_batch", ctypes.c_void_p),
        ("end_batch", ctypes.c_void_p),
        ("sync", ctypes.c_void_p),
    ]


def reference_scalar_backend():
    """The reference's compute_backend_scalar() vtable (compute_backend.c:101-117),
    or None when oracle/_ref was not built (no reference checkout)."""
    if not os.path.exists(_REF_PATH):
        return None
    L = ctypes.CDLL(_REF_PATH)
    L.compute_backend_scalar.restype = ctypes.POINTER(_RefBackend)
    return L.compute_backend_scalar().contents


# -- the reference's own single-token attention (oracle/_ref/libref_attention.so) -

_REF_ATTN_PATH = os.path.join(HERE, "_ref", "libref_attention.so")


class ReferenceAttention:
    """The reference MoE engine's attention_block (qwen_model.c:456-524) and
    RoPE table (qwen_model.c:346-353), driven through oracle/ref_attention.c
    on a model file written by oracle/ref_gguf.py.  F32 cache, NEOX RoPE over
    the whole head, no freq factors: it pins the semantics the oracle shares
    with it (GQA head mapping, scale, causal range, softmax, P.V, NEOX pairing,
    the angle schedule), not ggml's F16 roundings."""

    def __init__(self, path):
        L = ctypes.CDLL(path)
        L.ref_attention_step.restype = ctypes.c_int
        L.ref_attention_step.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, _f32p, _f32p, _f32p, _f32p,
                                         _f32p, ctypes.c_int, _f32p, _f32p, _f32p, _f32p, _f32p]
        L.ref_model_geometry.restype = ctypes.c_int
        L.ref_model_geometry.argtypes = [ctypes.c_char_p, ctypes.c_int] + [ctypes.POINTER(ctypes.c_int)] * 3 + \
            [ctypes.POINTER(ctypes.c_float)] * 2
        self._lib = L

    def geometry(self, gguf, max_seq):
        v = [ctypes.c_int() for _ in range(3)] + [ctypes.c_float() for _ in range(2)]
        rc = self._lib.ref_model_geometry(gguf.encode(), max_seq, *[ctypes.byref(x) for x in v])
        assert rc == 0, rc
        return tuple(x.value for x in v)

    def step(self, gguf, max_seq, pos, k_rows, v_rows, q, k, v, use_norm, n_head, n_head_kv, head_dim):
        """One decode step at `pos` over cache rows [pos][n_head_kv*head_dim] F32.
        Returns (attention output, stored K row, stored V row, cos table, sin table)."""
        nkvd = n_head_kv * head_dim
        kr = np.ascontiguousarray(np.asarray(k_rows, np.float32).reshape(pos, nkvd))
        vr = np.ascontiguousarray(np.asarray(v_rows, np.float32).reshape(pos, nkvd))
        q = np.ascontiguousarray(q, np.float32).reshape(-1)
        k = np.ascontiguousarray(k, np.float32).reshape(-1)
        v = np.ascontiguousarray(v, np.float32).reshape(-1)
        out = np.zeros(n_head * head_dim, np.float32)
        ko = np.zeros(nkvd, np.float32)
        vo = np.zeros(nkvd, np.float32)
        cs = np.zeros((max_seq, head_dim // 2), np.float32)
        sn = np.zeros((max_seq, head_dim // 2), np.float32)
        rc = self._lib.ref_attention_step(gguf.encode(), max_seq, pos, _p(kr), _p(vr), _p(q), _p(k), _p(v),
                                          int(use_norm), _p(out), _p(ko), _p(vo), _p(cs), _p(sn))
        assert rc == 0, rc
        return out, ko, vo, cs, sn


def reference_attention():
    """ReferenceAttention over oracle/_ref/libref_attention.so, or None when it
    was not built (no reference checkout on this host)."""
    if not os.path.exists(_REF_ATTN_PATH):
        return None
    return ReferenceAttention(_REF_ATTN_PATH)
