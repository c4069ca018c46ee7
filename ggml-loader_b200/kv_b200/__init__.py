"""Python binding of the B200 KV-cache append + attention library (ctypes over
the C ABI in include/kv_api.h and include/kv_bench.h).

The library (lib/libkv_b200.so) is the product; this module only marshals
arguments.  There is no fallback: if the shared library is missing or fails
to load, every entry point raises.
"""
import ctypes
import os

from . import specs, synth  # noqa: F401

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
# KV_B200_LIBRARY names another build of the same library to load instead
# (a measurement variant such as the phase-stamp build)
LIB_PATH = os.environ.get("KV_B200_LIBRARY") or os.path.join(PKG, "lib", "libkv_b200.so")

KV_OK = 0
KV_E_ARG = -1
KV_E_OOM = -2
KV_E_RANGE = -3
KV_E_CUDA = -4
KV_E_COMM = -5
KV_E_TIMEOUT = -6
KV_E_STATE = -7
KV_E_UNSUPPORTED = -8

KERNELS = {"append": 0, "attn": 1, "prefill": 2, "pfold": 3, "gather": 4, "prefill2": 5}

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_f32p = ctypes.POINTER(ctypes.c_float)


class KvConfig(ctypes.Structure):
    _fields_ = [
        ("n_layer", _i32), ("n_head", _i32), ("n_head_kv", _i32), ("head_dim", _i32), ("n_rot", _i32),
        ("rope_mode", _i32),
        ("rope_base", ctypes.c_float), ("rope_freq_scale", ctypes.c_float),
        ("rope_attn_factor", ctypes.c_float), ("rope_ext_factor", ctypes.c_float),
        ("rope_beta_fast", ctypes.c_float), ("rope_beta_slow", ctypes.c_float),
        ("n_ctx_orig", _i32),
        ("rope_freq_factors", _f32p),
        ("qk_norm", _i32), ("rms_eps", ctypes.c_float),
        ("n_ctx", _i64), ("n_ctx_train", _i64),
        ("longrope_clamp", _i32), ("n_batch_max", _i32), ("device", _i32),
        ("n_shards", _i32), ("shard", _i32),
        ("comm_id", _vp),
        ("ring_cells", _i64),
        ("flash_attn", _i32),
    ]


class KvError(RuntimeError):
    def __init__(self, code, what):
        self.code = code
        super().__init__("%s failed: %d (%s): %s" % (what, code, strerror(code), last_error()))


_lib = None


def lib():
    """Load lib/libkv_b200.so (raises if it is not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError("libkv_b200.so is not built (%s); run ggml-loader_b200/build.py "
                          "or __graft_entry__.build()" % LIB_PATH)
    L = ctypes.CDLL(LIB_PATH)
    cfgp = ctypes.POINTER(KvConfig)
    sig = {
        "kv_config_init": (ctypes.c_int, [cfgp]),
        "kv_cache_bytes": (_u64, [cfgp, _i64]),
        "kv_auto_n_ctx": (_i64, [cfgp, _i64]),
        "kv_alloc": (ctypes.c_int, [cfgp, ctypes.POINTER(_vp)]),
        "kv_free": (ctypes.c_int, [_vp]),
        "kv_n_ctx": (ctypes.c_int, [_vp, ctypes.POINTER(_i64)]),
        "kv_append": (ctypes.c_int, [_vp, _i32, _i64, _i32, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _vp]),
        "kv_append_bias": (ctypes.c_int, [_vp, _i32, _i64, _i32, _vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp,
                                          _vp, _vp, _vp, _vp]),
        "kv_attend": (ctypes.c_int, [_vp, _i32, _i64, _i32, _vp, _vp]),
        "kv_attend_mask": (ctypes.c_int, [_vp, _i32, _i64, _i32, _vp, _i32, _i64, ctypes.c_uint32, _vp, _vp]),
        "kv_forward": (ctypes.c_int, [_vp, _i64, _i32, _vp, _i64, _vp, _i64, _vp, _i64, _i64, _vp, _vp, _i64,
                                      _vp, _i64, _vp]),
        "kv_export_rows": (ctypes.c_int, [_vp, _i32, _i32, _i64, _i64, _vp]),
        "kv_import_rows": (ctypes.c_int, [_vp, _i32, _i32, _i64, _i64, _vp]),
        "kv_shard_info": (ctypes.c_int, [_vp] + [ctypes.POINTER(_i32)] * 4),
        "kv_comm_unique_id": (ctypes.c_int, [_vp]),
        "kv_strerror": (ctypes.c_char_p, [ctypes.c_int]),
        "kv_last_error": (ctypes.c_char_p, []),
        "kv_fill_synthetic": (ctypes.c_int, [_vp, _u64, _u64, _i64, _i64, _vp]),
        "kv_gen_normal_device": (ctypes.c_int, [_vp, _u64, _u64, _u64, _i64, _vp]),
        "kv_profile_enable": (ctypes.c_int, [_vp, ctypes.c_int]),
        "kv_profile_reset": (ctypes.c_int, [_vp]),
        "kv_profile_read": (ctypes.c_int, [_vp, _i32, ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_double)]),
        "kv_kernel_name": (ctypes.c_char_p, [_i32]),
        "kv_launch_count": (_i64, [_vp]),
        "kv_debug_stamps": (_i64, [_vp, _vp, ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
        "kv_attend_decode_noalloc": (ctypes.c_int, [_vp, _vp, _i32, _i32, _i32, _i64, _vp, _vp, _vp]),
        "kv_status": (ctypes.c_int, [_vp, _vp]),
        "kv_debug_inject": (ctypes.c_int, [_vp, _i32, _u64]),
        "kv_rope_table_host": (ctypes.c_int, [cfgp, _i64, _i64, _vp]),
        "kv_shard_geometry": (ctypes.c_int, [cfgp, _i32] + [ctypes.POINTER(_i32)] * 4),
        "kv_decode_ctas": (ctypes.c_int, [_i32, _i32, _i64, ctypes.POINTER(_i32)]),
        "kv_decode_grid_fits": (ctypes.c_int, [_i32, _i32, _i32]),
        "kv_decode_shape": (ctypes.c_int, [_i32, _i32, _i64, ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                                           ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name, None)
        if fn is None and os.environ.get("KV_B200_LIBRARY"):
            continue   # a measurement build of an earlier revision may lack newer entry points
        if fn is None:
            raise ImportError("%s does not export %s" % (LIB_PATH, name))
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def strerror(code):
    return lib().kv_strerror(code).decode()


def last_error():
    return lib().kv_last_error().decode()


def _check(rc, what):
    if rc != KV_OK:
        raise KvError(rc, what)
    return rc


def _ptr(x):
    """Device/host address of a torch tensor, numpy array, int or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    raise TypeError("cannot take the address of %r" % type(x))


def _stream(s):
    if s is None:
        return None
    if isinstance(s, int):
        return s
    return s.cuda_stream


def make_config(spec, n_ctx=None, n_batch_max=None, device=-1, n_shards=1, shard=0, comm_id=None, ring_cells=0,
                flash_attn=False):
    """A KvConfig from a specs.py dict.  Keeps referenced buffers alive on the
    returned object (freq factors, comm id).  ring_cells > 0 makes a ring cache
    (positions bounded by n_ctx, rows = ring_cells)."""
    import numpy as np
    c = KvConfig()
    lib().kv_config_init(ctypes.byref(c))
    c.n_layer = spec["n_layer"]
    c.n_head = spec["n_head"]
    c.n_head_kv = spec["n_head_kv"]
    c.head_dim = spec["head_dim"]
    c.n_rot = spec.get("n_rot", spec["head_dim"])
    c.rope_mode = spec.get("rope_mode", 2)
    c.rope_base = spec.get("rope_base", 10000.0)
    c.rope_freq_scale = spec.get("rope_freq_scale", 1.0)
    c.rope_attn_factor = spec.get("rope_attn_factor", 1.0)
    c.rope_ext_factor = spec.get("rope_ext_factor", 0.0)
    c.rope_beta_fast = spec.get("rope_beta_fast", 0.0)
    c.rope_beta_slow = spec.get("rope_beta_slow", 0.0)
    c.n_ctx_orig = spec.get("n_ctx_orig", 0)
    ff = spec.get("rope_freq_factors")
    c._ff = None if ff is None else np.ascontiguousarray(ff, dtype=np.float32)
    c.rope_freq_factors = None if c._ff is None else c._ff.ctypes.data_as(_f32p)
    c.qk_norm = int(spec.get("qk_norm") or 0)   # True -> 1 (RMSNorm); 2 = nGPT
    c.rms_eps = spec.get("rms_eps", 1e-6)
    c.n_ctx = spec.get("n_ctx", 0) if n_ctx is None else n_ctx
    c.n_ctx_train = spec.get("n_ctx_train", 0)
    c.longrope_clamp = 1 if spec.get("longrope_clamp") else 0
    c.n_batch_max = spec.get("n_batch_max", 512) if n_batch_max is None else n_batch_max
    c.device = device
    c.n_shards = n_shards
    c.shard = shard
    c.ring_cells = ring_cells
    c.flash_attn = 1 if flash_attn else 0
    if comm_id is not None:
        c._id = ctypes.create_string_buffer(bytes(comm_id), 128)
        c.comm_id = ctypes.cast(c._id, _vp)
    return c


def cache_bytes(cfg, n_ctx):
    return int(lib().kv_cache_bytes(ctypes.byref(cfg), n_ctx))


def auto_n_ctx(cfg, free_bytes):
    return int(lib().kv_auto_n_ctx(ctypes.byref(cfg), free_bytes))


def rope_table_host(cfg, pos0, npos):
    """The RoPE (cos, sin) table kv_alloc would upload, computed on the host."""
    import numpy as np
    out = np.zeros((npos, cfg.n_rot // 2, 2), np.float32)
    _check(lib().kv_rope_table_host(ctypes.byref(cfg), pos0, npos, out.ctypes.data), "kv_rope_table_host")
    return out


def shard_geometry(cfg, shard):
    vals = [_i32() for _ in range(4)]
    _check(lib().kv_shard_geometry(ctypes.byref(cfg), shard, *[ctypes.byref(v) for v in vals]),
           "kv_shard_geometry")
    return tuple(v.value for v in vals)


def comm_unique_id():
    buf = ctypes.create_string_buffer(128)
    _check(lib().kv_comm_unique_id(buf), "kv_comm_unique_id")
    return bytes(buf.raw)


class Context:
    """Owns one kv_ctx (the cache of every layer on one GPU / shard)."""

    def __init__(self, cfg):
        self.cfg = cfg
        h = _vp()
        _check(lib().kv_alloc(ctypes.byref(cfg), ctypes.byref(h)), "kv_alloc")
        self.h = h
        n = _i64()
        _check(lib().kv_n_ctx(self.h, ctypes.byref(n)), "kv_n_ctx")
        self.n_ctx = n.value
        vals = [_i32() for _ in range(4)]
        _check(lib().kv_shard_info(self.h, *[ctypes.byref(v) for v in vals]), "kv_shard_info")
        self.q_head0, self.n_q_heads, self.kv_head0, self.n_kv_heads = [v.value for v in vals]

    def close(self):
        if getattr(self, "h", None):
            lib().kv_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # -- the path ---------------------------------------------------------
    def append(self, layer, n_past, n_new, q, q_stride, k, k_stride, v, v_stride,
               q_norm_w=None, k_norm_w=None, stream=None):
        return _check(lib().kv_append(self.h, layer, n_past, n_new, _ptr(q), q_stride, _ptr(k), k_stride,
                                      _ptr(v), v_stride, _ptr(q_norm_w), _ptr(k_norm_w), _stream(stream)),
                      "kv_append")

    def append_bias(self, layer, n_past, n_new, q, q_stride, k, k_stride, v, v_stride,
                    q_norm_w=None, k_norm_w=None, q_bias=None, k_bias=None, v_bias=None, stream=None):
        """kv_append with the qwen2 QKV projection biases added in the load."""
        return _check(lib().kv_append_bias(self.h, layer, n_past, n_new, _ptr(q), q_stride, _ptr(k), k_stride,
                                           _ptr(v), v_stride, _ptr(q_norm_w), _ptr(k_norm_w), _ptr(q_bias),
                                           _ptr(k_bias), _ptr(v_bias), _stream(stream)),
                      "kv_append_bias")

    def attend(self, layer, n_past, n_new, out, stream=None):
        return _check(lib().kv_attend(self.h, layer, n_past, n_new, _ptr(out), _stream(stream)), "kv_attend")

    def attend_mask(self, layer, n_past, n_new, mask, out, flash=False, stream=None):
        """kv_attend with the caller's additive mask (a CUDA tensor of n_new rows,
        float32 or float16, row stride mask.stride(0); None = the implicit causal
        mask) and the flash-attn branch when flash is true."""
        mtype, mstride = 0, 0
        if mask is not None:
            import torch
            assert mask.dim() == 2 and mask.stride(1) == 1 and mask.dtype in (torch.float32, torch.float16)
            mtype, mstride = int(mask.dtype == torch.float16), mask.stride(0)
        return _check(lib().kv_attend_mask(self.h, layer, n_past, n_new, _ptr(mask), mtype, mstride,
                                           1 if flash else 0, _ptr(out), _stream(stream)), "kv_attend_mask")

    def forward(self, n_past, n_new, q, q_stride, k, k_stride, v, v_stride, in_layer_stride,
                q_norm_w, k_norm_w, norm_layer_stride, out, out_layer_stride, stream=None):
        return _check(lib().kv_forward(self.h, n_past, n_new, _ptr(q), q_stride, _ptr(k), k_stride, _ptr(v),
                                       v_stride, in_layer_stride, _ptr(q_norm_w), _ptr(k_norm_w),
                                       norm_layer_stride, _ptr(out), out_layer_stride, _stream(stream)),
                      "kv_forward")

    # -- rows ---------------------------------------------------------------
    def export_rows(self, layer, which, row0, nrows):
        import numpy as np
        d = self.cfg.head_dim
        out = np.empty((nrows, self.n_kv_heads, d), np.uint16)
        _check(lib().kv_export_rows(self.h, layer, which, row0, nrows, out.ctypes.data), "kv_export_rows")
        return out

    def import_rows(self, layer, which, row0, rows_u16):
        import numpy as np
        rows_u16 = np.ascontiguousarray(rows_u16, dtype=np.uint16)
        _check(lib().kv_import_rows(self.h, layer, which, row0, rows_u16.shape[0], rows_u16.ctypes.data),
               "kv_import_rows")

    # -- bench helpers ----------------------------------------------------
    def fill_synthetic(self, seed, row0, nrows, stream_base=synth.STREAM_CACHE, stream=None):
        return _check(lib().kv_fill_synthetic(self.h, seed, stream_base, row0, nrows, _stream(stream)),
                      "kv_fill_synthetic")

    def profile(self, on=True):
        _check(lib().kv_profile_enable(self.h, 1 if on else 0), "kv_profile_enable")

    def profile_reset(self):
        _check(lib().kv_profile_reset(self.h), "kv_profile_reset")

    def profile_read(self, kernel):
        n = _i64()
        ms = ctypes.c_double()
        kid = KERNELS[kernel] if isinstance(kernel, str) else kernel
        _check(lib().kv_profile_read(self.h, kid, ctypes.byref(n), ctypes.byref(ms)), "kv_profile_read")
        return n.value, ms.value

    def launch_count(self):
        return int(lib().kv_launch_count(self.h))

    def debug_stamps(self):
        """The phase-stamp build's ring of decode launches: (array [ring][max_cta][16]
        of %globaltimer values, launches stamped so far).  Other builds raise."""
        import numpy as np
        ring, mc = _i32(), _i32()
        n = int(lib().kv_debug_stamps(self.h, None, ctypes.byref(ring), ctypes.byref(mc)))
        if n < 0:
            _check(KV_E_UNSUPPORTED, "kv_debug_stamps")
        buf = np.zeros(ring.value * mc.value * 16, np.uint64)
        n = int(lib().kv_debug_stamps(self.h, buf.ctypes.data, ctypes.byref(ring), ctypes.byref(mc)))
        return buf.reshape(ring.value, mc.value, 16), n

    def status(self, stream=None):
        """KV_OK, or KV_E_TIMEOUT if a bounded device-side wait expired (raises)."""
        return _check(lib().kv_status(self.h, _stream(stream)), "kv_status")

    def debug_inject(self, what, limit_ns=0):
        _check(lib().kv_debug_inject(self.h, what, limit_ns), "kv_debug_inject")


def attend_decode_noalloc(k_cache, v_cache, n_head, n_head_kv, head_dim, n_kv, q, out, stream=None):
    """kv_attend_decode_noalloc: one token's decode attention over caller-owned
    buffers, with the library's fixed built-in scratch (no device allocation)."""
    return _check(lib().kv_attend_decode_noalloc(_ptr(k_cache), _ptr(v_cache), n_head, n_head_kv, head_dim, n_kv,
                                                 _ptr(q), _ptr(out), _stream(stream)),
                  "kv_attend_decode_noalloc")


def gen_normal_device(dst, seed, stream_id, n, idx0=0, stream=None):
    return _check(lib().kv_gen_normal_device(_ptr(dst), seed, stream_id, idx0, n, _stream(stream)),
                  "kv_gen_normal_device")
