"""The checkpoint loader (ditch_cuda_checkpoint_inspect /
ditch_cuda_model_load_checkpoint): a Hugging Face directory (config.json +
*.safetensors) or a GGUF file read in place, its tensors handed to the device
loader as stored, the way src/model.zig's load resolves names, layouts and
quantised formats (src/safetensors.zig, src/gguf.zig, src/moe.zig:83-92,
728-770). The files are written from the committed golden fixtures by
tests/checkpoint_files.py.

CPU: the config each file yields against the fixture's own spec, the tensor
count, and the refusals. GPU: a model loaded from the file against the model
built from the fixture's tensors through ditch_cuda_model_load, bit for bit
(deterministic K splits)."""
import json
import os
import struct

import numpy as np
import pytest

import ditch_b200
from checkpoint_files import (fixture, llama3_factors, write_gguf, write_gguf_fixture, write_gguf_from_hf,
                              write_gguf_with_package, write_hf_dir, write_llama_gguf)
from golden_loader import Golden
from oracle.model import flatten_batch

HF_FAMILIES = ["qwen2", "qwen2_fp8", "qwen2_int4", "qwen3", "llama", "mixtral", "qwen3_moe", "qwen3_moe_fused",
               "qwen3_moe_fused_t"]

# GGUF files converted from the bf16 Hugging Face fixtures (llama.cpp names,
# permuted llama q / k, stacked experts)
GGUF_FROM_HF = {"qwen2_bf16_gguf": "qwen2", "llama_gguf": "llama", "qwen3_gguf": "qwen3",
                "qwen3_moe_gguf": "qwen3_moe", "mixtral_gguf": "mixtral"}
FILES = HF_FAMILIES + ["qwen2_gguf", "llama_gguf_fixture", "qwen2_gguf_pkg", "llama_gguf_embedded",
                       "llama_gguf_rope_freqs"] + list(GGUF_FROM_HF)
# Llama 3's theta: with head_dim 8 its longest wavelength passes 8192 positions,
# so the largest factor is the scaling factor itself (how ditch recognises it)
LLAMA3_THETA = 500000.0
ROPE_KEYS = ("rope_scaling", "rope_factor", "rope_low_ff", "rope_high_ff", "rope_orig_max")

SPEC_KEYS = ["n_layers", "hidden", "heads", "kv_heads", "head_dim", "vocab", "qk_norm", "n_experts", "top_k",
             "moe_inter", "norm_topk", "moe_layers", "rope_scaling", "rope_factor", "rope_low_ff", "rope_high_ff",
             "rope_orig_max"]


def checkpoint(tmp_path, family):
    path = str(tmp_path / "model.gguf")
    if family == "qwen2_gguf":
        return write_gguf_fixture(path, family)
    if family == "llama_gguf_fixture":  # the reference's own llama GGUF fixture (per-frequency rope divisors)
        return write_gguf_fixture(path, "llama_gguf")
    if family == "qwen2_gguf_pkg":
        return write_gguf_with_package(path)
    if family == "llama_gguf_embedded":  # the HF config (llama3 rope included) inside the file
        return write_gguf_from_hf(path, "llama", embed_config=True, drop_rope_scaling=False)
    if family == "llama_gguf_rope_freqs":  # Llama 3's standard scaling as llama.cpp's factors
        c, _, _, _ = fixture("llama")
        f = llama3_factors(LLAMA3_THETA, c["head_dim"], 8.0)
        return write_llama_gguf(path, extra={"rope_freqs.weight": ("F32", f, [len(f)])}, rope_theta=LLAMA3_THETA)
    if family in GGUF_FROM_HF:
        return write_gguf_from_hf(path, GGUF_FROM_HF[family])
    return write_hf_dir(str(tmp_path / family), family)


def golden_spec(family):
    base = {"qwen2_gguf_pkg": "qwen2_gguf", "llama_gguf_embedded": "llama", "llama_gguf_rope_freqs": "llama",
            "llama_gguf_fixture": "llama_gguf"}
    g = Golden(base.get(family) or GGUF_FROM_HF.get(family) or family)
    s = dict(g.spec)
    if family in GGUF_FROM_HF:  # GGUF metadata carries no llama3 rope keys
        for k in ROPE_KEYS:
            s.pop(k, None)
    if family == "llama_gguf_rope_freqs":
        s.update(rope_scaling=1, rope_factor=8.0, rope_low_ff=1.0, rope_high_ff=4.0, rope_orig_max=8192.0,
                 rope_theta=LLAMA3_THETA)
    return g, s


def check_spec(got, want):
    for k in SPEC_KEYS:
        if k in want:
            assert got.get(k) == (int(want[k]) if isinstance(want[k], bool) else want[k]), k
    assert got.get("rope_scaling", 0) == int(want.get("rope_scaling", 0))
    if got.get("inter"):
        assert got["inter"] == want["inter"]
    assert got["eps"] == pytest.approx(want["eps"], rel=1e-6)
    assert got["rope_theta"] == pytest.approx(want["rope_theta"], rel=1e-6)


@pytest.mark.parametrize("family", FILES)
def test_inspect_matches_fixture_spec(tmp_path, family):
    path = checkpoint(tmp_path, family)
    spec, n = ditch_b200.inspect_checkpoint(path)
    g, want = golden_spec(family)
    check_spec(spec, want)
    # one table entry per canonical weight, stacked experts counted once
    n_want = sum(1 for c, hf in g.hf_names().items() if g.has(hf))
    n_want += 3 * sum(1 for x in (want.get("moe_layers") or []) if x)
    assert n == n_want


def test_own_gguf_writer_reads_back_with_the_package(tmp_path):
    """The test's GGUF writer checked by the `gguf` package's reader: names,
    ggml types, logical shapes and bytes."""
    gguf = pytest.importorskip("gguf")
    path = write_gguf_fixture(str(tmp_path / "m.gguf"), "qwen2_gguf")
    _, dtypes, shapes, raw = fixture("qwen2_gguf")
    r = gguf.GGUFReader(path)
    assert str(bytes(r.fields["general.architecture"].parts[-1]), "utf8") == "qwen2"
    seen = {}
    for t in r.tensors:
        seen[t.name] = t
        assert t.tensor_type.name == {"F16": "F16", "F32": "F32", "GGML_Q8_0": "Q8_0"}[dtypes[t.name]]
        want = shapes.get(t.name) or list(raw[t.name].shape)
        assert list(reversed([int(x) for x in t.shape])) == list(want)
        assert np.asarray(t.data).tobytes() == raw[t.name].tobytes()
    assert set(seen) == set(raw)


def test_hf_dir_with_shards(tmp_path):
    """A checkpoint split over several safetensors files, as large models are."""
    config, dtypes, _, raw = fixture("qwen2")
    from checkpoint_files import write_safetensors
    d = tmp_path / "sharded"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(config))
    names = sorted(raw)
    for i, part in enumerate((names[: len(names) // 2], names[len(names) // 2:])):
        write_safetensors(str(d / f"model-0000{i + 1}-of-00002.safetensors"), {n: (dtypes[n], raw[n]) for n in part})
    spec, n = ditch_b200.inspect_checkpoint(str(d))
    check_spec(spec, Golden("qwen2").spec)


def test_refusals(tmp_path):
    with pytest.raises(ditch_b200.DitchCudaError):
        ditch_b200.inspect_checkpoint(str(tmp_path / "missing"))
    # a model_type the device path does not take
    config, dtypes, _, raw = fixture("qwen2")
    d = write_hf_dir(str(tmp_path / "other"), "qwen2")
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(dict(config, model_type="gpt2"), f)
    with pytest.raises(ditch_b200.Unsupported):
        ditch_b200.inspect_checkpoint(d)
    # a required tensor missing
    d = write_hf_dir(str(tmp_path / "short"), "qwen2")
    from checkpoint_files import write_safetensors
    keep = {n: (dtypes[n], raw[n]) for n in sorted(raw) if "layers.1.mlp.up_proj" not in n}
    write_safetensors(os.path.join(d, "model.safetensors"), keep)
    with pytest.raises(ditch_b200.DitchCudaError, match="up_proj"):
        ditch_b200.inspect_checkpoint(d)
    # a safetensors header that points past the end of its file
    d = write_hf_dir(str(tmp_path / "trunc"), "qwen2")
    p = os.path.join(d, "model.safetensors")
    size = os.path.getsize(p)
    with open(p, "r+b") as f:
        f.truncate(size - 64)
    with pytest.raises(ditch_b200.DitchCudaError):
        ditch_b200.inspect_checkpoint(d)
    # not a GGUF file
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + bytes(60))
    with pytest.raises(ditch_b200.DitchCudaError):
        ditch_b200.inspect_checkpoint(str(bad))
    # a ggml type the device path has no decoder for (Q5_0 = 6)
    q = tmp_path / "q5.gguf"
    blob = np.zeros(22 * 2, np.uint8)
    from checkpoint_files import GGML_TYPE
    GGML_TYPE["Q5_0"] = 6
    try:
        write_gguf(str(q), "qwen2", [("qwen2.block_count", 4, 1)], {"token_embd.weight": ("Q5_0", blob, [2, 32])})
    finally:
        del GGML_TYPE["Q5_0"]
    with pytest.raises(ditch_b200.Unsupported):
        ditch_b200.inspect_checkpoint(str(q))


def test_gguf_rope_freqs(tmp_path):
    """rope_freqs.weight equal to Llama 3's standard scaling (low 1, high 4,
    8192 positions, any factor) becomes that scaling, as ditch recognises it
    (src/gguf_model.zig:311-326); any other factors are kept as per-frequency
    divisors (src/gguf_model.zig:227-228, 326-335)."""
    c, _, _, _ = fixture("llama")
    half = c["head_dim"] // 2
    ones = write_llama_gguf(str(tmp_path / "ones.gguf"),
                            extra={"rope_freqs.weight": ("F32", np.ones(half, np.float32), [half])})
    spec, _ = ditch_b200.inspect_checkpoint(ones)
    assert spec["rope_scaling"] == 1 and spec["rope_factor"] == 1.0  # factor 1: plain rope
    f = llama3_factors(LLAMA3_THETA, c["head_dim"], 32.0)
    std = write_llama_gguf(str(tmp_path / "std.gguf"), extra={"rope_freqs.weight": ("F32", f, [half])},
                           rope_theta=LLAMA3_THETA)
    spec, _ = ditch_b200.inspect_checkpoint(std)
    assert (spec["rope_scaling"], spec["rope_factor"], spec["rope_low_ff"], spec["rope_high_ff"],
            spec["rope_orig_max"]) == (1, 32.0, 1.0, 4.0, 8192.0)
    odd = np.arange(1, half + 1, dtype=np.float32)
    path = write_llama_gguf(str(tmp_path / "f.gguf"), extra={"rope_freqs.weight": ("F32", odd, [half])})
    spec, _ = ditch_b200.inspect_checkpoint(path)
    assert spec["rope_scaling"] == 4
    np.testing.assert_array_equal(spec["rope_factors"], odd)


def _rope_of(tmp_path, name, rope_scaling, **extra):
    config, _, _, _ = fixture("qwen2")
    d = write_hf_dir(str(tmp_path / name), "qwen2")
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(dict(config, rope_scaling=rope_scaling, **extra), f)
    return ditch_b200.inspect_checkpoint(d)[0]


def test_rope_scaling_types(tmp_path):
    """parseRopeScaling (src/arch.zig:1646-1720) for every type the reference
    reads: linear, yarn (with its default attention factor 0.1 ln(factor) + 1,
    arch.zig:1722-1725, or mscale / mscale_all_dim), longrope (the short
    factors, attention factor sqrt(1 + ln(factor) / ln(original))),
    ditch_factors; dynamic and unknown types read as plain RoPE."""
    f32 = lambda x: float(np.float32(x))
    s = _rope_of(tmp_path, "lin", {"rope_type": "linear", "factor": 2.5})
    assert (s["rope_scaling"], s["rope_factor"]) == (2, 2.5)
    s = _rope_of(tmp_path, "yarn", {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 2048})
    assert (s["rope_scaling"], s["rope_factor"], s["rope_orig_max"]) == (3, 4.0, 2048.0)
    assert (s["rope_beta_fast"], s["rope_beta_slow"], s["rope_truncate"]) == (32.0, 1.0, 1)
    assert s["rope_attention_factor"] == pytest.approx(f32(0.1 * np.log(np.float32(4.0)) + 1.0), rel=1e-7)
    s = _rope_of(tmp_path, "yarn2", {"type": "yarn", "factor": 40, "mscale": 1.0, "mscale_all_dim": 1.0,
                                     "beta_fast": 16, "beta_slow": 2, "truncate": False})
    assert s["rope_attention_factor"] == 1.0 and (s["rope_beta_fast"], s["rope_beta_slow"], s["rope_truncate"]) == \
        (16.0, 2.0, 0)
    half = fixture("qwen2")[0]["hidden_size"] // fixture("qwen2")[0]["num_attention_heads"] // 2
    short = [1.0 + 0.25 * i for i in range(half - 1)]  # one short: the last divisor stays 1
    s = _rope_of(tmp_path, "lr", {"rope_type": "longrope", "short_factor": short, "long_factor": [9.0] * half},
                 max_position_embeddings=8192, original_max_position_embeddings=2048)
    assert s["rope_scaling"] == 4
    np.testing.assert_array_equal(s["rope_factors"], np.asarray(short + [1.0], np.float32))
    assert s["rope_attention_factor"] == pytest.approx(np.sqrt(1 + np.log(4.0) / np.log(2048.0)), rel=1e-6)
    s = _rope_of(tmp_path, "df", {"rope_type": "ditch_factors", "factors": [1, 2, 3]})
    assert s["rope_scaling"] == 4
    np.testing.assert_array_equal(s["rope_factors"], np.asarray([1, 2, 3], np.float32))
    for name, rs in (("dyn", {"rope_type": "dynamic", "factor": 2.0}), ("unk", {"rope_type": "su", "factor": 2.0})):
        assert _rope_of(tmp_path, name, rs).get("rope_scaling", 0) == 0


def test_safetensors_header_is_parsed_not_trusted(tmp_path):
    """A header length larger than the file and a tensor whose byte range
    disagrees with its dtype x shape are errors, not reads out of bounds."""
    d = tmp_path / "h"
    d.mkdir()
    config, _, _, _ = fixture("qwen2")
    (d / "config.json").write_text(json.dumps(config))
    with open(d / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", 1 << 40) + b"{}")
    with pytest.raises(ditch_b200.DitchCudaError):
        ditch_b200.inspect_checkpoint(str(d))
    hdr = json.dumps({"model.embed_tokens.weight": {"dtype": "BF16", "shape": [4, 4], "data_offsets": [0, 30]}}).encode()
    with open(d / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(hdr)) + hdr + bytes(30))
    with pytest.raises(ditch_b200.DitchCudaError, match="holds 30 bytes"):
        ditch_b200.inspect_checkpoint(str(d))


# ---- on the device -----------------------------------------------------------

def _logits(m, prompts):
    toks, rb, rp, cap, first, take, last = flatten_batch(prompts)
    return m.forward(toks, rb, rp, (), last)[1]


@pytest.mark.gpu
@pytest.mark.parametrize("family", FILES)
def test_load_checkpoint_matches_tensor_table(device, tmp_path, family):
    """The model loaded from the file computes bit-identical logits to the one
    built from the fixture's own tensor table (which test_gpu_model checks
    against the reference's logits)."""
    path = checkpoint(tmp_path, family)
    g, spec = golden_spec(family)
    prompts = g.prompts()
    device.set_deterministic(True)
    try:
        a = ditch_b200.Model.from_checkpoint(device, path, max_seq=64)
        try:
            got = _logits(a, prompts)
        finally:
            a.close()
        b = ditch_b200.Model(device, spec, g.cuda_tensors(), max_seq=64)
        try:
            want = _logits(b, prompts)
        finally:
            b.close()
    finally:
        device.set_deterministic(False)
    assert got.shape == want.shape
    assert np.array_equal(got, want), float(np.abs(got - want).max())
