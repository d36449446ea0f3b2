"""A GGUF v2/v3 writer for tests (test infrastructure): metadata of every value type,
tensors of any ggml type id with caller-given bytes, optional general.alignment, and the
malformed variants the readers must reject."""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
        U64: "<Q", I64: "<q", F64: "<d"}


def _s(b: bytes | str) -> bytes:
    b = b.encode() if isinstance(b, str) else b
    return struct.pack("<Q", len(b)) + b


def _value(vtype, v) -> bytes:
    if vtype == STR:
        return _s(v)
    if vtype == ARR:
        et, items = v
        out = struct.pack("<IQ", et, len(items))
        return out + b"".join(_value(et, x) for x in items)
    return struct.pack(_FMT[vtype], v)


def build(kvs, tensors, version=3, alignment=None):
    """kvs: [(key, vtype, value)] (ARR value = (elem_type, items)); tensors:
    [(name, ggml_type, dims, data_bytes)] with dims[0] contiguous. Returns (file bytes,
    {name: absolute data offset})."""
    kvs = list(kvs)
    align = 32
    if alignment is not None:
        kvs.append(("general.alignment", U32, alignment))
        align = alignment
    head = struct.pack("<IIQQ", 0x46554747, version, len(tensors), len(kvs))
    head += b"".join(_s(k) + struct.pack("<I", t) + _value(t, v) for k, t, v in kvs)
    rel, off = [], 0
    for _, _, _, data in tensors:
        rel.append(off)
        off += (len(data) + align - 1) // align * align
    for (name, gt, dims, _), r in zip(tensors, rel):
        head += _s(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        head += struct.pack("<IQ", gt, r)
    data_off = (len(head) + align - 1) // align * align
    body = bytearray(head + b"\0" * (data_off - len(head)))
    for (_, _, _, data), r in zip(tensors, rel):
        body += b"\0" * (data_off + r - len(body)) + bytes(data)
    offsets = {t[0]: data_off + r for t, r in zip(tensors, rel)}
    return bytes(body), offsets


def sample_file(alignment=None, version=3, extra_tensors=()):
    """Metadata of every type and F32 / Q4_K / Q6_K / Q8_0 / unknown-type tensors."""
    rng = np.random.default_rng(5)
    kvs = [("general.architecture", STR, "qwen3"), ("qwen3.block_count", U32, 2),
           ("qwen3.rope.freq_base", F32, 1e6), ("general.flag", BOOL, 1), ("t.u8", U8, 200),
           ("t.i8", I8, -5), ("t.u16", U16, 60000), ("t.i16", I16, -30000), ("t.i32", I32, -7),
           ("t.u64", U64, 1 << 40), ("t.i64", I64, -(1 << 40)), ("t.f64", F64, 0.125),
           ("tokenizer.ggml.tokens", ARR, (STR, ["a", "bb", "ccc"])),
           ("test.nums", ARR, (I32, [10, 20, 30])), ("test.u8s", ARR, (U8, [1, 2, 250]))]
    tensors = [("odd.weight", 200, (16,), b"\1" * 16),
               ("f32.weight", 0, (8, 3), rng.normal(0, 1, 24).astype(np.float32).tobytes()),
               ("q4k.weight", 12, (512, 3), rng.integers(0, 256, 2 * 144 * 3, dtype=np.uint8).tobytes()),
               ("q6k.weight", 14, (256, 5), rng.integers(0, 256, 210 * 5, dtype=np.uint8).tobytes()),
               ("q80.weight", 8, (64, 2), rng.integers(0, 256, 2 * 34 * 2, dtype=np.uint8).tobytes())
               ] + list(extra_tensors)
    return build(kvs, tensors, version=version, alignment=alignment)


def malformed():
    """(reason, file bytes) pairs every reader must reject."""
    good, _ = sample_file()
    out = [("bad magic", b"X" + good[1:]),
           ("bad version", good[:4] + struct.pack("<I", 99) + good[8:]),
           ("truncated", good[:-8])]
    far, _ = build([], [("t0", 0, (4, 2), np.zeros(8, np.float32).tobytes())])
    # patch the single tensor's offset (last 8 bytes of its entry) far past the end
    i = far.index(b"t0") + 2 + 4 + 16 + 4
    out.append(("out-of-range offset", far[:i] + struct.pack("<Q", 1 << 40) + far[i + 8:]))
    nested = struct.pack("<IIQQ", 0x46554747, 3, 0, 1) + _s("bad") + struct.pack("<IIQ", ARR, ARR, 1)
    out.append(("nested array", nested))
    return out


def gpt2_byte_tokens():
    """The 256 single-byte tokens of a GPT-2 style byte-level vocabulary (the public
    byte -> unicode convention: printable bytes map to themselves, the others to 256 + n)."""
    direct = set(range(33, 127)) | set(range(161, 173)) | set(range(174, 256))
    out, n = [], 0
    for b in range(256):
        if b in direct:
            out.append(chr(b))
        else:
            out.append(chr(256 + n))
            n += 1
    return out


def dense_model_file(port, cfg, seed=0, std=0.02, byte_vocab=False):
    """A Qwen3-layout dense model (llama.cpp tensor names) with weights ~ N(0, std) encoded
    by the oracle's encoder: Q4_K, with Q6_K attn_v / ffn_down / output; fp32 norms.
    byte_vocab: the first 256 tokens are the GPT-2 byte tokens, so a byte-level tokenizer
    (the reference's) encodes any prompt without merges."""
    from oracle.oracle import Q4_K, Q6_K
    rng = np.random.default_rng(seed)
    H, F, NH, NKV, HD = cfg.hidden, cfg.ffn, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim

    def mat(qt, rows, cols):
        return (qt, (cols, rows), port.quantize(qt, rng.normal(0, std, (rows, cols)).astype(np.float32)).tobytes())

    def norm(n):
        return (0, (n,), (1.0 + 0.1 * rng.normal(0, 1, n)).astype(np.float32).tobytes())

    ts = [("token_embd.weight",) + mat(Q4_K, cfg.vocab, H)]
    for l in range(cfg.n_layers):
        p = f"blk.{l}."
        ts += [(p + "attn_norm.weight",) + norm(H), (p + "attn_q.weight",) + mat(Q4_K, NH * HD, H),
               (p + "attn_k.weight",) + mat(Q4_K, NKV * HD, H), (p + "attn_v.weight",) + mat(Q6_K, NKV * HD, H),
               (p + "attn_output.weight",) + mat(Q4_K, H, NH * HD), (p + "attn_q_norm.weight",) + norm(HD),
               (p + "attn_k_norm.weight",) + norm(HD), (p + "ffn_norm.weight",) + norm(H),
               (p + "ffn_gate.weight",) + mat(Q4_K, F, H), (p + "ffn_up.weight",) + mat(Q4_K, F, H),
               (p + "ffn_down.weight",) + mat(Q6_K, H, F)]
    ts += [("output_norm.weight",) + norm(H), ("output.weight",) + mat(Q6_K, cfg.vocab, H)]
    kvs = [("general.architecture", STR, "qwen3"), ("qwen3.block_count", U32, cfg.n_layers),
           ("qwen3.embedding_length", U32, H), ("qwen3.feed_forward_length", U32, F),
           ("qwen3.attention.head_count", U32, NH), ("qwen3.attention.head_count_kv", U32, NKV),
           ("qwen3.attention.key_length", U32, HD), ("qwen3.context_length", U32, cfg.kv_cap),
           ("qwen3.rope.freq_base", F32, cfg.rope_theta),
           ("qwen3.attention.layer_norm_rms_epsilon", F32, cfg.rms_eps),
           ("tokenizer.ggml.tokens", ARR, (STR, (gpt2_byte_tokens() if byte_vocab else []) +
                                             [f"t{i}" for i in range(256 if byte_vocab else 0, cfg.vocab)]))]
    if byte_vocab:
        kvs.append(("tokenizer.ggml.model", STR, "gpt2"))
    return build(kvs, [(n, t, d, b) for n, t, d, b in ts])


def hybrid_model_file(port, cfg, seed=0, std=0.02):
    """A qwen35moe-architecture hybrid MoE model (llama.cpp tensor names and layout) for a
    katali_lab_b200.synth.HybridConfig: Gated DeltaNet layers (attn_qkv, attn_gate, ssm_beta,
    ssm_alpha, ssm_out, ssm_conv1d, ssm_a = -exp(A_log), ssm_dt.bias, ssm_norm) and gated
    attention layers (attn_q with query and gate rows per head, attn_k, attn_v, attn_output,
    attn_q_norm, attn_k_norm), each followed by the routed experts (ffn_gate_inp fp32 router,
    ffn_gate_exps / ffn_up_exps [hidden, ffn, experts] Q4_K, ffn_down_exps [ffn, hidden,
    experts] Q6_K). Matrices ~ N(0, std) encoded by the oracle's encoder (the types of
    synth.HYBRID_TYPES); norms 1 + 0.1 N(0, 1), conv taps N(0, 0.3), A_log = log U(1, 16),
    dt_bias U(-4, -2)."""
    from oracle.oracle import Q4_K, Q6_K
    rng = np.random.default_rng(seed)
    H, E, F = cfg.hidden, cfg.n_experts, cfg.ffn
    nk, nv, dh, ck = cfg.ssm_k_heads, cfg.ssm_v_heads, cfg.ssm_head_dim, cfg.ssm_conv
    Cc, VD = (2 * nk + nv) * dh, nv * dh
    QD, KD = cfg.n_heads * cfg.head_dim, cfg.n_kv_heads * cfg.head_dim

    def enc(qt, rows, cols):
        return port.quantize(qt, rng.normal(0, std, (rows, cols)).astype(np.float32)).tobytes()

    def mat(qt, rows, cols):
        return (qt, (cols, rows), enc(qt, rows, cols))

    def f32(dims, a):
        return (0, dims, np.ascontiguousarray(a, dtype=np.float32).tobytes())

    def norm(n):
        return f32((n,), 1.0 + 0.1 * rng.normal(0, 1, n))

    ts = [("token_embd.weight",) + mat(Q4_K, cfg.vocab, H)]
    for l in range(cfg.n_layers):
        p = f"blk.{l}."
        ts += [(p + "attn_norm.weight",) + norm(H)]
        if cfg.kind(l) == 0:
            a_log = np.log(rng.uniform(1.0, 16.0, nv)).astype(np.float32)
            ts += [(p + "attn_qkv.weight",) + mat(Q4_K, Cc, H), (p + "attn_gate.weight",) + mat(Q4_K, VD, H),
                   (p + "ssm_beta.weight",) + mat(Q4_K, nv, H), (p + "ssm_alpha.weight",) + mat(Q4_K, nv, H),
                   (p + "ssm_out.weight",) + mat(Q4_K, H, VD),
                   (p + "ssm_conv1d.weight",) + f32((ck, Cc), rng.normal(0, 0.3, (Cc, ck))),
                   (p + "ssm_a",) + f32((nv,), -np.exp(a_log)),
                   (p + "ssm_dt.bias",) + f32((nv,), rng.uniform(-4.0, -2.0, nv)),
                   (p + "ssm_norm.weight",) + norm(dh)]
        else:
            ts += [(p + "attn_q.weight",) + mat(Q4_K, 2 * QD, H), (p + "attn_k.weight",) + mat(Q4_K, KD, H),
                   (p + "attn_v.weight",) + mat(Q6_K, KD, H), (p + "attn_output.weight",) + mat(Q4_K, H, QD),
                   (p + "attn_q_norm.weight",) + norm(cfg.head_dim),
                   (p + "attn_k_norm.weight",) + norm(cfg.head_dim)]
        ts += [(p + "post_attention_norm.weight",) + norm(H),
               (p + "ffn_gate_inp.weight",) + f32((H, E), rng.normal(0, std, (E, H))),
               (p + "ffn_gate_exps.weight", Q4_K, (H, F, E), b"".join(enc(Q4_K, F, H) for _ in range(E))),
               (p + "ffn_up_exps.weight", Q4_K, (H, F, E), b"".join(enc(Q4_K, F, H) for _ in range(E))),
               (p + "ffn_down_exps.weight", Q6_K, (F, H, E), b"".join(enc(Q6_K, H, F) for _ in range(E)))]
    ts += [("output_norm.weight",) + norm(H), ("output.weight",) + mat(Q6_K, cfg.vocab, H)]
    A = "qwen35moe"
    kvs = [("general.architecture", STR, A), (A + ".block_count", U32, cfg.n_layers),
           (A + ".embedding_length", U32, H), (A + ".attention.head_count", U32, cfg.n_heads),
           (A + ".attention.head_count_kv", U32, cfg.n_kv_heads),
           (A + ".attention.key_length", U32, cfg.head_dim), (A + ".rope.dimension_count", U32, cfg.rope_dim),
           (A + ".rope.freq_base", F32, cfg.rope_theta),
           (A + ".attention.layer_norm_rms_epsilon", F32, cfg.rms_eps),
           (A + ".expert_count", U32, E), (A + ".expert_used_count", U32, cfg.top_k),
           (A + ".expert_feed_forward_length", U32, F), (A + ".ssm.conv_kernel", U32, ck),
           (A + ".ssm.state_size", U32, dh), (A + ".ssm.group_count", U32, nk),
           (A + ".ssm.time_step_rank", U32, nv), (A + ".ssm.inner_size", U32, VD),
           (A + ".full_attention_interval", U32, cfg.attn_every), (A + ".context_length", U32, cfg.kv_cap),
           ("tokenizer.ggml.tokens", ARR, (STR, [f"t{i}" for i in range(cfg.vocab)]))]
    return build(kvs, [(n, t, d, b) for n, t, d, b in ts])
