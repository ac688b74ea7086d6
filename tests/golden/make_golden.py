"""Generates the golden fixtures under tests/golden/ from the reference's own
fixture models and reference outputs.

Run in a container where the reference checkout is mounted:

    python tests/golden/make_golden.py /path/to/ditch/tests/fixtures

For every family it writes ``<family>.npz`` holding the raw tensors of the
tiny checkpoint exactly as stored on disk (bf16 as uint16 bits, F8_E4M3
codes as uint8, packed INT words as int32, ...), the config.json text, and
the reference cases: token ids, last-token logits and the last-token
residual of every layer entry (``reference.json``, checked by the reference
at 2e-3 max abs in src/model_test.zig:58-84). The GPU box never reads the
reference tree; the tests read only these .npz files.
"""
import json
import os
import struct
import sys

import numpy as np

FAMILIES = ["qwen2", "llama", "qwen3", "qwen3_moe", "qwen2_fp8", "qwen2_int4", "qwen3_moe_big", "qwen3_moe_fused",
            "qwen3_moe_fused_t", "mixtral"]

DTYPES = {
    "BF16": np.uint16,
    "F16": np.uint16,
    "F32": np.float32,
    "F8_E4M3": np.uint8,
    "I32": np.int32,
    "I64": np.int64,
    "U8": np.uint8,
}


def read_safetensors(path):
    """Raw tensors of one safetensors file (own parser: numpy has no fp8)."""
    out = {}
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        base = 8 + n
        for name, meta in header.items():
            if name == "__metadata__":
                continue
            a, b = meta["data_offsets"]
            f.seek(base + a)
            raw = f.read(b - a)
            arr = np.frombuffer(raw, dtype=DTYPES[meta["dtype"]]).reshape(meta["shape"])
            out[name] = (meta["dtype"], arr.copy())
    return out


# ggml type -> (name, elements per block, bytes per block)
GGML = {0: ("F32", 1, 4), 1: ("F16", 1, 2), 8: ("GGML_Q8_0", 32, 34), 12: ("GGML_Q4_K", 256, 144),
        14: ("GGML_Q6_K", 256, 210), 30: ("BF16", 1, 2)}
GGUF_FAMILIES = ["qwen2_gguf", "llama_gguf"]


def read_gguf(path):
    """Metadata and raw tensors of a GGUF v3 file (own parser). A tensor of
    ggml dims (cols, rows) is returned as [rows][row bytes] of uint8 for block
    types, or as the typed [rows][cols] array (f16 / bf16 as uint16 bits)."""
    def rd(f, fmt):
        return struct.unpack("<" + fmt, f.read(struct.calcsize("<" + fmt)))

    def rstr(f):
        n, = rd(f, "Q")
        return f.read(n).decode("utf-8", "replace")

    scalar = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}

    def rval(f, t):
        if t == 8:
            return rstr(f)
        if t == 9:
            at, = rd(f, "I")
            n, = rd(f, "Q")
            return [rval(f, at) for _ in range(n)]
        return rd(f, scalar[t])[0]

    with open(path, "rb") as f:
        assert f.read(4) == b"GGUF"
        _version, = rd(f, "I")
        nt, = rd(f, "Q")
        nkv, = rd(f, "Q")
        meta = {}
        for _ in range(nkv):
            k = rstr(f)
            t, = rd(f, "I")
            meta[k] = rval(f, t)
        infos = []
        for _ in range(nt):
            name = rstr(f)
            nd, = rd(f, "I")
            dims = rd(f, "Q" * nd)
            typ, = rd(f, "I")
            off, = rd(f, "Q")
            infos.append((name, dims, typ, off))
        align = meta.get("general.alignment", 32)
        base = (f.tell() + align - 1) // align * align
        out = {}
        for name, dims, typ, off in infos:
            tname, per, nbytes = GGML[typ]
            cols = dims[0]
            rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
            row_bytes = cols // per * nbytes
            f.seek(base + off)
            raw = np.frombuffer(f.read(rows * row_bytes), np.uint8)
            if tname == "F32":
                arr = raw.view(np.float32).reshape(rows, cols) if len(dims) > 1 else raw.view(np.float32)
            elif tname in ("F16", "BF16"):
                arr = raw.view(np.uint16).reshape(rows, cols) if len(dims) > 1 else raw.view(np.uint16)
            else:
                arr = raw.reshape(rows, row_bytes)
            out[name] = (tname, arr.copy(), (rows, cols))
    return meta, out


def gguf_config(meta, tensors):
    """An HF-style config.json from the GGUF metadata (the fields the forward needs)."""
    a = meta["general.architecture"]
    cfg = {"model_type": a, "gguf": True, "hidden_size": meta[f"{a}.embedding_length"],
           "intermediate_size": meta[f"{a}.feed_forward_length"], "num_hidden_layers": meta[f"{a}.block_count"],
           "num_attention_heads": meta[f"{a}.attention.head_count"],
           "num_key_value_heads": meta.get(f"{a}.attention.head_count_kv", meta[f"{a}.attention.head_count"]),
           "rms_norm_eps": meta[f"{a}.attention.layer_norm_rms_epsilon"],
           "rope_theta": meta.get(f"{a}.rope.freq_base", 10000.0),
           "vocab_size": tensors["token_embd.weight"][2][0],
           "tie_word_embeddings": "output.weight" not in tensors}
    if f"{a}.attention.key_length" in meta:
        cfg["head_dim"] = meta[f"{a}.attention.key_length"]
    return cfg


def main(fixtures):
    here = os.path.dirname(os.path.abspath(__file__))
    for fam in FAMILIES:
        d = os.path.join(fixtures, fam)
        tensors = {}
        for fn in sorted(os.listdir(d)):
            if fn.endswith(".safetensors"):
                tensors.update(read_safetensors(os.path.join(d, fn)))
        cfg = open(os.path.join(d, "config.json")).read()
        ref = json.load(open(os.path.join(d, "reference.json")))
        payload = {"config_json": np.frombuffer(cfg.encode(), np.uint8)}
        dtypes = {}
        for name, (dt, arr) in tensors.items():
            payload["t/" + name] = arr
            dtypes[name] = dt
        payload["dtypes_json"] = np.frombuffer(json.dumps(dtypes).encode(), np.uint8)
        for i, case in enumerate(ref["cases"]):
            payload[f"case{i}/ids"] = np.asarray(case["ids"], np.uint32)
            payload[f"case{i}/last_logits"] = np.asarray(case["last_logits"], np.float32)
            payload[f"case{i}/last_hidden"] = np.asarray(case["last_hidden"], np.float32)
            payload[f"case{i}/argmax"] = np.asarray([case["argmax"]], np.int64)
        payload["n_cases"] = np.asarray([len(ref["cases"])], np.int64)
        np.savez_compressed(os.path.join(here, fam + ".npz"), **payload)
        print(fam, len(tensors), "tensors", len(ref["cases"]), "cases")
    for fam in GGUF_FAMILIES:
        d = os.path.join(fixtures, fam)
        meta, tensors = read_gguf(os.path.join(d, "model.gguf"))
        cfg = json.dumps(gguf_config(meta, tensors))
        ref = json.load(open(os.path.join(d, "reference.json")))
        payload = {"config_json": np.frombuffer(cfg.encode(), np.uint8)}
        dtypes, shapes = {}, {}
        for name, (dt, arr, shape) in tensors.items():
            payload["t/" + name] = arr
            dtypes[name] = dt
            shapes[name] = shape
        payload["dtypes_json"] = np.frombuffer(json.dumps(dtypes).encode(), np.uint8)
        payload["shapes_json"] = np.frombuffer(json.dumps(shapes).encode(), np.uint8)
        for i, case in enumerate(ref["cases"]):
            payload[f"case{i}/ids"] = np.asarray(case["ids"], np.uint32)
            payload[f"case{i}/last_logits"] = np.asarray(case["last_logits"], np.float32)
            payload[f"case{i}/last_hidden"] = np.asarray(case["last_hidden"], np.float32)
            payload[f"case{i}/argmax"] = np.asarray([case["argmax"]], np.int64)
        payload["n_cases"] = np.asarray([len(ref["cases"])], np.int64)
        np.savez_compressed(os.path.join(here, fam + ".npz"), **payload)
        print(fam, len(tensors), "tensors (gguf)", len(ref["cases"]), "cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <ditch checkout>/tests/fixtures")
    main(sys.argv[1])
