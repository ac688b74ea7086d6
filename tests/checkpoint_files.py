"""Writes the committed golden fixtures back to checkpoint files (a Hugging
Face directory of config.json + model.safetensors, or a GGUF v3 file), the
inputs of the library's checkpoint loader. The tensors are the fixtures' own
stored bytes under their original names and layouts (mixtral's w1 / w2 / w3,
fused and transposed-fused experts, FP8 codes with their scale_inv,
pack-quantized INT groups, ggml blocks)."""
import json
import os
import struct

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

NP_DTYPE = {"BF16": np.uint16, "F16": np.uint16, "F32": np.float32, "F8_E4M3": np.uint8, "I32": np.int32,
            "I64": np.int64, "U8": np.uint8}


def fixture(family):
    z = np.load(os.path.join(GOLDEN, family + ".npz"))
    config = json.loads(bytes(z["config_json"]).decode())
    dtypes = json.loads(bytes(z["dtypes_json"]).decode())
    shapes = json.loads(bytes(z["shapes_json"]).decode()) if "shapes_json" in z.files else {}
    raw = {k[2:]: z[k] for k in z.files if k.startswith("t/")}
    return config, dtypes, shapes, raw


def write_safetensors(path, tensors):
    """tensors: name -> (dtype string, numpy array of the stored bytes)."""
    header, blobs, off = {}, [], 0
    for name, (dt, a) in tensors.items():
        b = np.ascontiguousarray(a).tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_hf_dir(directory, family):
    config, dtypes, _, raw = fixture(family)
    os.makedirs(directory, exist_ok=True)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(config, f)
    write_safetensors(os.path.join(directory, "model.safetensors"),
                      {n: (dtypes[n], raw[n]) for n in sorted(raw)})
    return directory


GGML_TYPE = {"F32": 0, "F16": 1, "GGML_Q8_0": 8, "GGML_Q4_K": 12, "BF16": 30}


def _gstr(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, arch, meta, tensors):
    """tensors: name -> (ggml dtype string, raw bytes array, [rows, cols] or [n])."""
    kv = [("general.architecture", 8, arch), ("general.alignment", 4, 32)] + meta
    out = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kv)))
    for key, ty, val in kv:
        out += _gstr(key) + struct.pack("<I", ty)
        out += _gstr(val) if ty == 8 else struct.pack({4: "<I", 5: "<i", 6: "<f"}[ty], val)
    off, blobs = 0, []
    for name, (dt, a, shape) in tensors.items():
        b = np.ascontiguousarray(a).tobytes()
        dims = list(reversed(shape))  # ggml: innermost first
        out += _gstr(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", GGML_TYPE[dt], off)
        blobs.append(b)
        off += (len(b) + 31) // 32 * 32
    out += b"\0" * ((32 - len(out) % 32) % 32)
    for b in blobs:
        out += b + b"\0" * ((32 - len(b) % 32) % 32)
    with open(path, "wb") as f:
        f.write(out)
    return path


def write_gguf_fixture(path, family):
    """A GGUF family of the fixtures (qwen2_gguf) as its own GGUF file."""
    config, dtypes, shapes, raw = fixture(family)
    meta = _meta(config, "qwen2")
    tensors = {}
    for n in sorted(raw):
        shp = shapes.get(n) or list(raw[n].shape)
        tensors[n] = (dtypes[n], raw[n], shp)
    return write_gguf(path, "qwen2", meta, tensors)


def _meta(config, arch):
    c = config
    return [(f"{arch}.block_count", 4, c["num_hidden_layers"]), (f"{arch}.embedding_length", 4, c["hidden_size"]),
            (f"{arch}.feed_forward_length", 4, c["intermediate_size"]),
            (f"{arch}.attention.head_count", 4, c["num_attention_heads"]),
            (f"{arch}.attention.head_count_kv", 4, c["num_key_value_heads"]),
            (f"{arch}.attention.layer_norm_rms_epsilon", 6, c["rms_norm_eps"]),
            (f"{arch}.rope.freq_base", 6, c["rope_theta"])]


def permute_qk(w, n_head):
    """llama.cpp's converter order of q / k rows: per head, (i, half) pairs."""
    rows = w.shape[0]
    return w.reshape(n_head, 2, rows // n_head // 2, *w.shape[1:]).swapaxes(1, 2).reshape(w.shape)


def write_llama_gguf(path, family="llama", extra=None):
    """A llama-layout fixture as a GGUF file of its own bf16 tensors, q / k
    rows permuted as llama.cpp's converter stores them. GGUF has no
    rope_scaling key (llama3 factors come as rope_freqs.weight, which the
    loader refuses), so the file carries plain rope. `extra`: more tensors,
    name -> (ggml dtype, array, shape)."""
    config, dtypes, _, raw = fixture(family)
    names = {"model.embed_tokens.weight": "token_embd.weight", "model.norm.weight": "output_norm.weight"}
    if "lm_head.weight" in raw:
        names["lm_head.weight"] = "output.weight"
    for i in range(config["num_hidden_layers"]):
        p, q = f"model.layers.{i}.", f"blk.{i}."
        names.update({p + "input_layernorm.weight": q + "attn_norm.weight",
                      p + "post_attention_layernorm.weight": q + "ffn_norm.weight",
                      p + "self_attn.q_proj.weight": q + "attn_q.weight", p + "self_attn.k_proj.weight": q + "attn_k.weight",
                      p + "self_attn.v_proj.weight": q + "attn_v.weight",
                      p + "self_attn.o_proj.weight": q + "attn_output.weight",
                      p + "mlp.gate_proj.weight": q + "ffn_gate.weight", p + "mlp.up_proj.weight": q + "ffn_up.weight",
                      p + "mlp.down_proj.weight": q + "ffn_down.weight"})
    tensors = {}
    for hf, gg in names.items():
        a = raw[hf]
        if gg.endswith("attn_q.weight"):
            a = permute_qk(a, config["num_attention_heads"])
        if gg.endswith("attn_k.weight"):
            a = permute_qk(a, config["num_key_value_heads"])
        tensors[gg] = (dtypes[hf], a, list(a.shape))
    tensors.update(extra or {})
    return write_gguf(path, "llama", _meta(config, "llama"), tensors)
