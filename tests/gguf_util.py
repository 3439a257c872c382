"""Test helpers: GGUF files written the way the reference's shards are
(candle's gguf_file::write via quantize_shard, src/quantize.rs:112-152:
version 3, no metadata, 32-byte alignment, dims innermost first) and the
reference's shard directory layout (src/streaming_quantized.rs:451-501)."""
import struct

import numpy as np

F32, F16, Q4_0, Q3_K, Q4_K, BF16 = 0, 1, 2, 11, 12, 30
LINEAR_NAMES = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


def _s(b: bytes) -> bytes:
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, tensors, metadata=(), alignment=32, version=3):
    """tensors: (name, ggml_type, shape outermost first, raw bytes)."""
    out = bytearray(b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(metadata)))
    for key, (vtype, value) in metadata:
        out += _s(key.encode()) + struct.pack("<I", vtype)
        if vtype == 8:
            out += _s(value.encode())
        elif vtype == 4:
            out += struct.pack("<I", value)
        elif vtype == 9:  # array of u32
            out += struct.pack("<IQ", 4, len(value)) + b"".join(struct.pack("<I", v) for v in value)
        else:
            raise ValueError(vtype)
    offs, off = [], 0
    for _, _, _, raw in tensors:
        offs.append(off)
        off += (len(raw) + alignment - 1) // alignment * alignment
    for (name, t, shape, _), o in zip(tensors, offs):
        out += _s(name.encode()) + struct.pack("<I", len(shape))
        out += b"".join(struct.pack("<Q", d) for d in reversed(shape))
        out += struct.pack("<IQ", t, o)
    out += b"\0" * ((-len(out)) % alignment)
    for (_, _, _, raw), o in zip(tensors, offs):
        out += bytes(raw) + b"\0" * ((-len(raw)) % alignment)
    with open(path, "wb") as f:
        f.write(out)


def write_shard_dir(d, cfg, qtype, host):
    """host: random_model(..., host_blocks=True)'s dict (single rank).  Norms
    are stored F16 as the reference's quantizer keeps them; returns the f32
    norms as the file holds them (f16-rounded)."""
    import os
    os.makedirs(d, exist_ok=True)
    rounded = []
    for l, (blocks, r1, r2) in enumerate(host["layers"]):
        p = f"model.layers.{l}."
        ts = []
        from rustyllm_b200.llama import layer_shapes
        for k, ((o, i), b) in enumerate(zip(layer_shapes(cfg), blocks)):
            ts.append((p + LINEAR_NAMES[k] + ".weight", qtype, (o, i), np.ascontiguousarray(b).tobytes()))
        n1, n2 = np.float16(r1), np.float16(r2)
        ts.append((p + "input_layernorm.weight", F16, (cfg["hidden"],), n1.tobytes()))
        ts.append((p + "post_attention_layernorm.weight", F16, (cfg["hidden"],), n2.tobytes()))
        write_gguf(os.path.join(d, f"model.layers.{l}.gguf"), ts)
        rounded.append((blocks, n1.astype(np.float32), n2.astype(np.float32)))
    V, H = cfg["vocab"], cfg["hidden"]
    write_gguf(os.path.join(d, "model.embed_tokens.gguf"),
               [("model.embed_tokens.weight", F16, (V, H), np.float16(host["embed"]).tobytes())])
    lnf = np.float16(host["ln_f"])
    write_gguf(os.path.join(d, "model.norm.gguf"), [("model.norm.weight", F16, (H,), lnf.tobytes())])
    write_gguf(os.path.join(d, "lm_head.gguf"),
               [("lm_head.weight", F16, (V, H), np.float16(host["lm_head"]).tobytes())])
    return rounded, lnf.astype(np.float32)
