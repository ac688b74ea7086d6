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
    """A GGUF family of the fixtures (qwen2_gguf, llama_gguf: its q / k rows in
    llama.cpp's order and its rope_freqs.weight, as stored) as its own GGUF file."""
    config, dtypes, shapes, raw = fixture(family)
    arch = config["model_type"]
    meta = _meta(config, arch)
    tensors = {}
    for n in sorted(raw):
        shp = shapes.get(n) or list(raw[n].shape)
        tensors[n] = (dtypes[n], raw[n], shp)
    return write_gguf(path, arch, meta, tensors)


def _meta(config, arch):
    c = config
    m = [(f"{arch}.block_count", 4, c["num_hidden_layers"]), (f"{arch}.embedding_length", 4, c["hidden_size"]),
         (f"{arch}.feed_forward_length", 4, c["intermediate_size"]),
         (f"{arch}.attention.head_count", 4, c["num_attention_heads"]),
         (f"{arch}.attention.head_count_kv", 4, c["num_key_value_heads"]),
         (f"{arch}.attention.layer_norm_rms_epsilon", 6, c["rms_norm_eps"]),
         (f"{arch}.rope.freq_base", 6, c["rope_theta"])]
    if c.get("head_dim"):
        m.append((f"{arch}.attention.key_length", 4, c["head_dim"]))
    return m


def permute_qk(w, n_head):
    """llama.cpp's converter order of q / k rows: per head, (i, half) pairs."""
    rows = w.shape[0]
    return w.reshape(n_head, 2, rows // n_head // 2, *w.shape[1:]).swapaxes(1, 2).reshape(w.shape)


GGUF_ARCH = {"llama": "llama", "mixtral": "llama", "qwen2": "qwen2", "qwen3": "qwen3", "qwen3_moe": "qwen3moe"}


def write_gguf_from_hf(path, family, extra=None, embed_config=False, drop_rope_scaling=True, rope_theta=None):
    """A bf16 Hugging Face fixture as a GGUF file of its own tensors under
    llama.cpp's names: q / k rows (and biases) permuted for the llama family,
    routed experts stacked into [E][rows][cols] `ffn_*_exps` tensors, the
    router as `ffn_gate_inp`. GGUF metadata has no llama3 rope keys (the
    factors come as rope_freqs.weight), so with `drop_rope_scaling` the file
    carries plain rope; `embed_config` stores the Hugging Face config as
    `ditch.hf.config_json`, as ditch's own export does. `extra`: more tensors,
    name -> (ggml dtype, array, shape); `rope_theta` replaces the fixture's."""
    config, dtypes, _, raw = fixture(family)
    if rope_theta is not None:
        config = dict(config, rope_theta=rope_theta)
    mt = config["model_type"]
    arch = GGUF_ARCH[mt]
    permuted = arch == "llama"
    L = config["num_hidden_layers"]
    out = {}

    def put(gg, hf, heads=None):
        a = raw[hf]
        if heads:
            a = permute_qk(a, heads)
        out[gg] = (dtypes[hf], a, list(a.shape))

    put("token_embd.weight", "model.embed_tokens.weight")
    put("output_norm.weight", "model.norm.weight")
    if "lm_head.weight" in raw:
        put("output.weight", "lm_head.weight")
    for i in range(L):
        p, q = f"model.layers.{i}.", f"blk.{i}."
        put(q + "attn_norm.weight", p + "input_layernorm.weight")
        put(q + "ffn_norm.weight", p + "post_attention_layernorm.weight")
        for a, b in (("q", "q_proj"), ("k", "k_proj"), ("v", "v_proj")):
            heads = (config["num_attention_heads"] if a == "q" else config["num_key_value_heads"]) \
                if permuted and a != "v" else None
            for kind in ("weight", "bias"):
                if p + f"self_attn.{b}.{kind}" in raw:
                    put(q + f"attn_{a}.{kind}", p + f"self_attn.{b}.{kind}", heads)
        put(q + "attn_output.weight", p + "self_attn.o_proj.weight")
        if p + "self_attn.q_norm.weight" in raw:
            put(q + "attn_q_norm.weight", p + "self_attn.q_norm.weight")
            put(q + "attn_k_norm.weight", p + "self_attn.k_norm.weight")
        moe = p + "block_sparse_moe.gate.weight" if mt == "mixtral" else p + "mlp.gate.weight"
        if moe in raw:
            put(q + "ffn_gate_inp.weight", moe)
            E = config.get("num_local_experts") or config["num_experts"]
            for proj, hf_proj in (("gate", "gate_proj"), ("up", "up_proj"), ("down", "down_proj")):
                if mt == "mixtral":
                    hf_proj = {"gate_proj": "w1", "up_proj": "w3", "down_proj": "w2"}[hf_proj]
                    names = [p + f"block_sparse_moe.experts.{e}.{hf_proj}.weight" for e in range(E)]
                else:
                    names = [p + f"mlp.experts.{e}.{hf_proj}.weight" for e in range(E)]
                st = np.stack([raw[n] for n in names])
                out[q + f"ffn_{proj}_exps.weight"] = (dtypes[names[0]], st, list(st.shape))
        else:
            for proj in ("gate", "up", "down"):
                put(q + f"ffn_{proj}.weight", p + f"mlp.{proj}_proj.weight")
    out.update(extra or {})
    meta = _meta(config, arch)
    if mt in ("mixtral", "qwen3_moe"):
        E = config.get("num_local_experts") or config["num_experts"]
        meta += [(f"{arch}.expert_count", 4, E), (f"{arch}.expert_used_count", 4, config["num_experts_per_tok"])]
        if mt == "qwen3_moe":
            meta.append((f"{arch}.expert_feed_forward_length", 4, config["moe_intermediate_size"]))
    if embed_config:
        c = dict(config)
        if drop_rope_scaling:
            c.pop("rope_scaling", None)
        meta.append(("ditch.hf.config_json", 8, json.dumps(c)))
    return write_gguf(path, arch, meta, out)


def write_llama_gguf(path, family="llama", extra=None, rope_theta=None):
    return write_gguf_from_hf(path, family, extra=extra, rope_theta=rope_theta)


def llama3_factors(theta, head_dim, factor, low_ff=1.0, high_ff=4.0, orig=8192.0):
    """llama.cpp's rope_freqs.weight for a llama3 rope scaling (its
    converter's generate_extra_tensors), in f32."""
    out = np.empty(head_dim // 2, np.float32)
    low_w, high_w = np.float32(orig / low_ff), np.float32(orig / high_ff)
    for i in range(head_dim // 2):
        freq = 1.0 / theta ** (2 * i / head_dim)
        wl = np.float32(2 * np.pi / freq)
        if wl < high_w:
            out[i] = 1.0
        elif wl > low_w:
            out[i] = factor
        else:
            sm = (np.float32(orig) / wl - np.float32(low_ff)) / np.float32(high_ff - low_ff)
            out[i] = 1.0 / ((1.0 - sm) / np.float32(factor) + sm)
    return out


def write_gguf_with_package(path, family="qwen2_gguf"):
    """The same fixture written by the `gguf` package's own GGUFWriter, an
    independent writer of the format."""
    import gguf
    config, dtypes, shapes, raw = fixture(family)
    c = config
    w = gguf.GGUFWriter(path, "qwen2")
    w.add_block_count(c["num_hidden_layers"])
    w.add_embedding_length(c["hidden_size"])
    w.add_feed_forward_length(c["intermediate_size"])
    w.add_head_count(c["num_attention_heads"])
    w.add_head_count_kv(c["num_key_value_heads"])
    w.add_layer_norm_rms_eps(c["rms_norm_eps"])
    w.add_rope_freq_base(c["rope_theta"])
    q = gguf.GGMLQuantizationType
    for n in sorted(raw):
        dt, a = dtypes[n], raw[n]
        if dt == "F16":
            w.add_tensor(n, a.view(np.float16))
        elif dt == "F32":
            w.add_tensor(n, a.astype(np.float32))
        else:
            rows = shapes[n][0]  # the package takes [rows][bytes per row]
            w.add_tensor(n, a.view(np.uint8).reshape(rows, -1), raw_dtype={"GGML_Q8_0": q.Q8_0, "GGML_Q4_K": q.Q4_K}[dt])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return path
