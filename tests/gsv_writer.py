"""Writes GSV1 weight containers (the format of the reference's
tools/convert.py:3-28) for the loader tests: little-endian header (magic,
version 1, flags bit 0 = fp16 segments present, name, config JSON, tensor
count), one directory entry per tensor (name, rank, dims, source dtype,
fp32 and fp16 segment offsets and sizes), then every fp32 block and every
fp16 block, each starting on a 64-byte boundary.

Test infrastructure: builds synthetic files; no checkpoint is converted.
"""
import json
import struct

import numpy as np

ALIGN = 64


def t2s_tensors(model: dict):
    """The reference's AR tensor names (t2s_engine.cpp:565-630) for a model
    from workloads.t2s_model: (name, fp32 array, fp16 bits or None)."""
    L, D, F, V = model["n_layers"], model["d_model"], model["ffn"], model["vocab"]
    h = lambda a: a.view(np.float16).astype(np.float32)  # noqa: E731
    out = []
    for i in range(L):
        p, ps = f"h.layers.{i}.", f"h.layers.{i}.self_attn."
        out += [(ps + "in_proj_weight", h(model["wqkv"][i]), model["wqkv"][i]),
                (ps + "in_proj_bias", model["bqkv"][i], None),
                (ps + "out_proj.weight", h(model["wout"][i]), model["wout"][i]),
                (ps + "out_proj.bias", model["bout"][i], None),
                (p + "linear1.weight", h(model["w1"][i]), model["w1"][i]),
                (p + "linear1.bias", model["b1"][i], None),
                (p + "linear2.weight", h(model["w2"][i]), model["w2"][i]),
                (p + "linear2.bias", model["b2"][i], None),
                (p + "norm1.weight", model["n1g"][i], None), (p + "norm1.bias", model["n1b"][i], None),
                (p + "norm2.weight", model["n2g"][i], None), (p + "norm2.bias", model["n2b"][i], None)]
    out += [("ar_predict_layer.weight", h(model["wpred"]), model["wpred"]),
            ("ar_audio_embedding.word_embeddings.weight", h(model["audio_emb"]), model["audio_emb"]),
            ("ar_audio_position.alpha", np.array([model["alpha_audio"]], np.float32), None)]
    config = {"meta": {"source": "synthetic"},
              "model_config": {"model": {"hidden_dim": D, "embedding_dim": D,
                                         "head": model["n_heads"], "linear_units": F,
                                         "n_layer": L, "vocab_size": V, "EOS": V - 1,
                                         "phoneme_vocab_size": 732}}}
    return out, config


def write(path, name: str, config: dict, tensors, slim=False, patch=None):
    """tensors: (name, fp32 array, fp16 bits or None).  slim: omit the fp32
    copy of tensors that have an fp16 one.  patch(entries) may edit the
    directory fields before they are written (negative tests)."""
    cfg = json.dumps(config).encode()
    nm = name.encode()
    head = b"GSV1" + struct.pack("<II", 1, 0) + struct.pack("<H", len(nm)) + nm
    head += struct.pack("<I", len(cfg)) + cfg + struct.pack("<I", len(tensors))
    entries = []
    for tname, f32, f16 in tensors:
        f32 = np.ascontiguousarray(f32, np.float32)
        entries.append(dict(name=tname.encode(), dims=list(f32.shape), dtype=2 if f16 is not None else 1,
                            f32=None if (slim and f16 is not None) else f32.tobytes(),
                            f16=None if f16 is None else np.ascontiguousarray(f16, np.uint16).tobytes()))
    dir_size = sum(2 + len(e["name"]) + 2 + 4 * len(e["dims"]) + 2 + 32 for e in entries)
    off = -(-(len(head) + dir_size) // ALIGN) * ALIGN
    blobs = []
    for kind in ("f32", "f16"):
        for e in entries:
            data = e[kind]
            e[kind + "_off"], e[kind + "_n"] = (off, len(data)) if data else (0, 0)
            if data:
                blobs.append((off, data))
                off = -(-(off + len(data)) // ALIGN) * ALIGN
    flags = 1 if any(e["f16"] for e in entries) else 0
    for e in entries:
        e["flags"] = flags
    if patch:
        patch(entries)
    flags = entries[0].get("flags", flags) if entries else flags
    head = head[:8] + struct.pack("<I", flags) + head[12:]
    d = b""
    for e in entries:
        d += struct.pack("<H", len(e["name"])) + e["name"] + struct.pack("<H", len(e["dims"]))
        d += struct.pack(f"<{len(e['dims'])}I", *e["dims"]) + struct.pack("<H", e["dtype"])
        d += struct.pack("<QQQQ", e["f32_off"], e["f32_n"], e["f16_off"], e["f16_n"])
    size = max([o + len(b) for o, b in blobs] + [len(head) + len(d)])
    buf = bytearray(size)
    buf[:len(head)] = head
    buf[len(head):len(head) + len(d)] = d
    for o, b in blobs:
        buf[o:o + len(b)] = b
    with open(path, "wb") as f:
        f.write(bytes(buf))
