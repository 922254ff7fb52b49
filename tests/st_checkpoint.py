"""Test helper: writes safetensors files, and a synth.Model as a checkpoint
under the tensor names the reference's loader looks up (ds_ocr.c:608-690):
per-expert gate/up/down matrices, separate embeddings, norms."""
import json
import os

import numpy as np

_DT = {"BF16": 2, "F16": 2, "F32": 4, "I32": 4, "I64": 8, "BOOL": 1}


def write_safetensors(path, tensors, metadata=None, pad_header=0):
    """tensors: {name: (dtype_str, np.ndarray)}; BF16 arrays as uint16."""
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, (dt, arr) in tensors.items():
        a = np.ascontiguousarray(arr)
        b = a.tobytes()
        assert len(b) == a.size * _DT[dt], name
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode() + b" " * pad_header
    with open(path, "wb") as f:
        f.write(np.uint64(len(h)).tobytes())
        f.write(h)
        for b in blobs:
            f.write(b)


def decoder_tensors(model, embed=None, tied=False, norm_dtype="BF16"):
    """{name: (dtype, array)} of a synth.Model in the reference's naming."""
    d = model.d
    H, I, S, E = d.hidden, d.moe_inter, d.shared_inter, d.n_experts

    def norm(v):
        v = np.asarray(v, np.float32)
        if norm_dtype == "F32":
            return ("F32", v)
        return ("BF16", (v.view(np.uint32) >> 16).astype(np.uint16))  # exact for the 1.0 norms

    t = {}
    t["model.embed_tokens.weight"] = ("BF16", model.lm_head if embed is None else embed)
    for l, lw in enumerate(model.layers):
        p = f"model.layers.{l}."
        t[p + "self_attn.q_proj.weight"] = ("BF16", lw.wq)
        t[p + "self_attn.k_proj.weight"] = ("BF16", lw.wk)
        t[p + "self_attn.v_proj.weight"] = ("BF16", lw.wv)
        t[p + "self_attn.o_proj.weight"] = ("BF16", lw.wo)
        t[p + "input_layernorm.weight"] = norm(lw.input_norm)
        t[p + "post_attention_layernorm.weight"] = norm(lw.post_norm)
        if lw.moe is None:
            t[p + "mlp.gate_proj.weight"] = ("BF16", lw.dense_gate)
            t[p + "mlp.up_proj.weight"] = ("BF16", lw.dense_up)
            t[p + "mlp.down_proj.weight"] = ("BF16", lw.dense_down)
            continue
        m = lw.moe
        t[p + "mlp.gate.weight"] = ("BF16", m.router)
        for e in range(E):
            gu = m.expert_gate_up(e).reshape(2 * I, H)
            t[p + f"mlp.experts.{e}.gate_proj.weight"] = ("BF16", gu[:I])
            t[p + f"mlp.experts.{e}.up_proj.weight"] = ("BF16", gu[I:])
            t[p + f"mlp.experts.{e}.down_proj.weight"] = ("BF16", m.expert_down(e).reshape(H, I))
        sgu = m.shared_gate_up().reshape(2 * S, H)
        t[p + "mlp.shared_experts.gate_proj.weight"] = ("BF16", sgu[:S])
        t[p + "mlp.shared_experts.up_proj.weight"] = ("BF16", sgu[S:])
        t[p + "mlp.shared_experts.down_proj.weight"] = ("BF16", m.shared_down)
    t["model.norm.weight"] = norm(model.final_norm)
    if not tied:
        t["lm_head.weight"] = ("BF16", model.lm_head)
    return t


def write_checkpoint(model, directory, shards=1, embed=None, tied=False, norm_dtype="BF16"):
    """One model.safetensors, or `shards` model-0000k-of-0000n files."""
    os.makedirs(directory, exist_ok=True)
    t = decoder_tensors(model, embed, tied, norm_dtype)
    names = list(t)
    if shards == 1:
        write_safetensors(os.path.join(directory, "model.safetensors"), t, metadata={"format": "pt"})
        return
    for k in range(shards):
        part = {n: t[n] for n in names[k::shards]}
        write_safetensors(os.path.join(directory, f"model-{k + 1:05d}-of-{shards:05d}.safetensors"), part,
                          metadata={"format": "pt"})
