"""Minimal GGUF model file for the reference-attention harness (oracle/ref_attention.c).

TEST INFRASTRUCTURE ONLY.  The harness loads a model through the reference's
own qwen_load() (src/moe_stream/qwen_model.c:211-367), which reads a GGUF file
with gguf_index_load() (src/moe_stream/gguf_index.c:189-321) and builds the
expert plan with moe_plan_build() (gguf_index.c:397-).  This writes the
smallest file those accept for a one-layer model with the attention geometry
under test: the metadata keys gguf_index_load reads, and every tensor
qwen_load and moe_plan_build look up, in F32 (GGUF type 0).  The projection
weights are zeros -- the harness's matmul returns the test's rows instead --
and the Q/K norm weights carry the test's gamma.

GGUF v3 layout (little endian): "GGUF", u32 version, u64 tensor count, u64
key/value count; each key a u64-length string, a u32 type and the value
(4 = u32, 6 = f32, 8 = string); each tensor info a name, u32 n_dims, u64 dims
(ne0 first), u32 type and u64 offset into the data section, which starts at
the next multiple of general.alignment.
"""
import struct

import numpy as np

_ALIGN = 32


def _str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write(path, n_head, n_head_kv, head_dim, rope_theta, eps=1e-6, q_norm=None, k_norm=None, n_embd=64,
          n_ff=32, n_expert=2, n_vocab=8):
    """Write the model file; q_norm / k_norm are the [head_dim] Q/K norm gammas
    (ones when None)."""
    arch = "qwen3moe"
    kv = [
        ("general.architecture", 8, arch),
        ("general.alignment", 4, _ALIGN),
        (arch + ".block_count", 4, 1),
        (arch + ".embedding_length", 4, n_embd),
        (arch + ".expert_feed_forward_length", 4, n_ff),
        (arch + ".expert_count", 4, n_expert),
        (arch + ".expert_used_count", 4, 1),
        (arch + ".attention.head_count", 4, n_head),
        (arch + ".attention.head_count_kv", 4, n_head_kv),
        (arch + ".attention.key_length", 4, head_dim),
        (arch + ".rope.freq_base", 6, float(rope_theta)),
        (arch + ".attention.layer_norm_rms_epsilon", 6, float(eps)),
    ]
    ones = np.ones(head_dim, np.float32)
    qn = ones if q_norm is None else np.asarray(q_norm, np.float32)
    kn = ones if k_norm is None else np.asarray(k_norm, np.float32)
    z = lambda *dims: np.zeros(int(np.prod(dims)), np.float32)
    tensors = [
        ("token_embd.weight", (n_embd, n_vocab), z(n_embd, n_vocab)),
        ("output_norm.weight", (n_embd,), np.ones(n_embd, np.float32)),
        ("output.weight", (n_embd, n_vocab), z(n_embd, n_vocab)),
        ("blk.0.attn_norm.weight", (n_embd,), np.ones(n_embd, np.float32)),
        ("blk.0.attn_q.weight", (n_embd, n_head * head_dim), z(n_embd, n_head * head_dim)),
        ("blk.0.attn_k.weight", (n_embd, n_head_kv * head_dim), z(n_embd, n_head_kv * head_dim)),
        ("blk.0.attn_v.weight", (n_embd, n_head_kv * head_dim), z(n_embd, n_head_kv * head_dim)),
        ("blk.0.attn_output.weight", (n_head * head_dim, n_embd), z(n_head * head_dim, n_embd)),
        ("blk.0.attn_q_norm.weight", (head_dim,), qn),
        ("blk.0.attn_k_norm.weight", (head_dim,), kn),
        ("blk.0.ffn_norm.weight", (n_embd,), np.ones(n_embd, np.float32)),
        ("blk.0.ffn_gate_inp.weight", (n_embd, n_expert), z(n_embd, n_expert)),
        ("blk.0.ffn_gate_exps.weight", (n_embd, n_ff, n_expert), z(n_embd, n_ff, n_expert)),
        ("blk.0.ffn_up_exps.weight", (n_embd, n_ff, n_expert), z(n_embd, n_ff, n_expert)),
        ("blk.0.ffn_down_exps.weight", (n_ff, n_embd, n_expert), z(n_ff, n_embd, n_expert)),
    ]
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv))
    for key, t, val in kv:
        head += _str(key) + struct.pack("<I", t)
        if t == 8:
            head += _str(val)
        elif t == 4:
            head += struct.pack("<I", val)
        else:
            head += struct.pack("<f", val)
    off = 0
    blobs = []
    for name, dims, data in tensors:
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", 0, off)
        blob = np.ascontiguousarray(data, np.float32).tobytes()
        pad = (-len(blob)) % _ALIGN
        blobs.append(blob + b"\0" * pad)
        off += len(blob) + pad
    head += b"\0" * ((-len(head)) % _ALIGN)
    with open(path, "wb") as f:
        f.write(head)
        for b in blobs:
            f.write(b)
    return path
