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

FAMILIES = ["qwen2", "llama", "qwen3", "qwen3_moe", "qwen2_fp8", "qwen2_int4"]

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


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <ditch checkout>/tests/fixtures")
    main(sys.argv[1])
