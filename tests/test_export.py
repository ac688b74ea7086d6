"""Export of an edited model (ditch_cuda_export_checkpoint, src/export.zig):
the source checkpoint written again with the deltas merged on the device.

CPU: the config.json rewrites against the reference's own test vectors
(src/dequant.zig:1312-1329, src/export.zig:291-300) and the loader's refusal
of an unfinished export. GPU: every exported tensor against the oracle's
merge (src/export.zig:88-131, src/moe.zig:368-390) of the source values and
the model's own deltas, bit for bit: edited weights merged and rounded,
decoded FP8 / INT groups, untouched tensors byte-identical; shards, index,
marker and side files; the reloaded export against the edited model."""
import json
import os
import struct

import numpy as np
import pytest

import ditch_b200
import oracle
from checkpoint_files import fixture, write_gguf_fixture, write_hf_dir
from golden_loader import Golden
from oracle.model import flatten_batch

ST_NP = {"BF16": np.uint16, "F16": np.uint16, "F32": np.float32, "I32": np.int32, "I64": np.int64,
         "F8_E4M3": np.uint8, "U8": np.uint8}


def read_dir(d):
    """name -> (dtype, shape, array of the stored bytes) over every shard."""
    out = {}
    for f in sorted(os.listdir(d)):
        if not f.endswith(".safetensors"):
            continue
        data = open(os.path.join(d, f), "rb").read()
        n = struct.unpack("<Q", data[:8])[0]
        h = json.loads(data[8:8 + n])
        assert list(h)[0] == "__metadata__"
        for name, e in h.items():
            if name == "__metadata__":
                continue
            a, b = e["data_offsets"]
            arr = np.frombuffer(data[8 + n + a:8 + n + b], ST_NP[e["dtype"]]).reshape(e["shape"])
            out[name] = (e["dtype"], e["shape"], arr)
    return out


# ---- CPU: config.json text --------------------------------------------------

STRIP_CASES = [  # src/dequant.zig:1312-1329
    ('{"a": 1, "quantization_config": {"quant_method": "fp8", "weight_block_size": [128, 128]}, "b": "x"}',
     '{"a": 1, "b": "x"}'),
    ('{\n  "a": 1,\n  "quantization_config": {"m": "}"}\n}', '{\n  "a": 1\n}'),
    ('{"text_config": {"quantization_config": [1, 2], "x": 2}, "quantization_config": null}',
     '{"text_config": {"x": 2}}'),
    ('{"no_quantization_config": 1}', '{"no_quantization_config": 1}'),
    ('{"expert_dtype": "fp4", "hc_mult": 4, "quantization_config": {"quant_method": "fp8"}}', '{"hc_mult": 4}'),
]


@pytest.mark.parametrize("src,want", STRIP_CASES)
def test_strip_quantization_config(src, want):
    assert ditch_b200.export_config(src, strip_quantization_config=True) == want


def test_config_dtype():
    """src/export.zig:291-300: every float dtype / torch_dtype value renamed,
    other values and look-alike strings untouched."""
    src = ('{"dtype": "bfloat16", "text_config": {"torch_dtype":"bfloat16", "model_type": "x"},\n'
           ' "quantization_config": {"dtype": "int8"}, "name": "dtype", "note": "a \\"dtype\\": \\"bfloat16\\" in a string"}')
    want = ('{"dtype": "float32", "text_config": {"torch_dtype":"float32", "model_type": "x"},\n'
            ' "quantization_config": {"dtype": "int8"}, "name": "dtype", "note": "a \\"dtype\\": \\"bfloat16\\" in a string"}')
    assert ditch_b200.export_config(src, dtype="f32") == want
    assert ditch_b200.export_config(src) == src


def test_unfinished_export_is_refused(tmp_path):
    d = write_hf_dir(str(tmp_path / "x"), "qwen2")
    ditch_b200.inspect_checkpoint(d)
    open(os.path.join(d, ".incomplete"), "w").write("export in progress\n")
    with pytest.raises(ditch_b200.DitchCudaError, match="incomplete"):
        ditch_b200.inspect_checkpoint(d)


def test_oracle_merge_forms_agree():
    """The row and column merges are one edit in two layouts (up to rounding)."""
    rng = np.random.default_rng(3)
    w = rng.standard_normal((6, 5)).astype(np.float32)
    a = rng.standard_normal((2, 5)).astype(np.float32)
    b = rng.standard_normal((6, 2)).astype(np.float32)
    rows = oracle.export_merge_rows(w, a, b)
    cols = oracle.export_merge_cols(w.T, a, b).T
    np.testing.assert_allclose(rows, cols, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(rows, w + b @ a, rtol=1e-6, atol=1e-6)


# ---- on the device -------------------------------------------------------------

def source_values(family):
    """name in the export -> (f32 values as the reference's store hands them
    out, the dtype they are stored in)."""
    config, dtypes, _, raw = fixture(family)
    q = config.get("quantization_config") or {}
    out = {}
    for n, a in raw.items():
        dt = dtypes[n]
        if n.endswith("_scale_inv") or any(n.endswith(s) for s in (".weight_scale", ".weight_zero_point",
                                                                    ".weight_shape", ".weight_g_idx")):
            continue
        if dt == "F8_E4M3":
            br, bc = q["weight_block_size"]
            out[n] = (oracle.bf16_bits_to_f32(oracle.dequant_fp8(a, raw[n + "_scale_inv"], br, bc)), "BF16")
        elif n.endswith(".weight_packed"):
            base = n[: -len("_packed")]
            rows, cols = (int(v) for v in raw[base + "_shape"])
            w = q["config_groups"]["group_0"]["weights"]
            sc = oracle.bf16_bits_to_f32(raw[base + "_scale"]) if dtypes[base + "_scale"] == "BF16" else raw[base + "_scale"]
            bits = oracle.dequant_int_packed(a, sc, raw.get(base + "_zero_point"), rows, cols, w["num_bits"],
                                             w["group_size"])
            out[base] = (oracle.bf16_bits_to_f32(bits), "BF16")
        elif dt == "BF16":
            out[n] = (oracle.bf16_bits_to_f32(a), "BF16")
        elif dt == "F16":
            out[n] = (a.view(np.float16).astype(np.float32), "F16")
        elif dt == "F32":
            out[n] = (a.astype(np.float32), "F32")
    return config, dtypes, raw, out


def edited(m, spec, name):
    """The model's delta on tensor `name`: (a, b, layout) or None."""
    parts = name.split(".")
    if not name.startswith("model.layers."):
        return None
    li = int(parts[2])
    rest = ".".join(parts[3:])
    moe = bool(spec.get("moe_layers") and spec["moe_layers"][li])
    if rest == "self_attn.o_proj.weight":
        d = m.delta(li, "attn_o_proj")
        return d and (*d, "rows")
    if rest == "mlp.down_proj.weight" and not moe:
        d = m.delta(li, "mlp_down_proj")
        return d and (*d, "rows")
    if moe and ((rest.startswith("mlp.experts.") and rest.endswith(".down_proj.weight")) or rest.endswith(".w2.weight")):
        e = int(parts[-3])
        d = m.delta(li, "expert_down_proj", e)
        return d and (*d, "rows")
    if moe and rest == "mlp.experts.down_proj":
        return [m.delta(li, "expert_down_proj", e) for e in range(spec["n_experts"])], None, "fused"
    return None


def expected_values(m, spec, name, vals):
    """f32 values of `name` after the oracle's merge of the model's delta."""
    d = edited(m, spec, name)
    if d is None:
        return vals, False
    if d[2] == "rows":
        return oracle.export_merge_rows(vals, d[0], d[1]), True
    out = np.array(vals, np.float32, copy=True)
    H, mi = spec["hidden"], spec["moe_inter"]
    transposed = out.shape[1] != H
    any_edit = False
    for e, de in enumerate(d[0]):
        if de is None:
            continue
        any_edit = True
        out[e] = oracle.export_merge_cols(out[e], *de) if transposed else oracle.export_merge_rows(out[e], *de)
    assert out.shape[1:] == ((mi, H) if transposed else (H, mi))
    return out, any_edit


def edit_model(m, spec, seed=5):
    rng = np.random.default_rng(seed)
    dirs = rng.standard_normal((spec["n_layers"] + 1, spec["hidden"])).astype(np.float32)
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    m.set_directions(dirs)
    po, pd = (1.2, 1.0, 0.5, 3.0), (1.0, 1.0, 0.4, 3.0)
    if spec.get("moe_layers"):
        m.apply_expert_edit(po, pd, n_experts=2, strength=0.8)
    else:
        m.apply_edit(po, pd)


def _logits(m, prompts):
    toks, rb, rp, cap, first, take, last = flatten_batch(prompts)
    return m.forward(toks, rb, rp, (), last)[1]


EXPORT_FAMILIES = ["qwen2", "qwen2_fp8", "qwen2_int4", "qwen3", "llama", "mixtral", "qwen3_moe", "qwen3_moe_fused",
                   "qwen3_moe_fused_t"]


@pytest.mark.gpu
@pytest.mark.parametrize("family", EXPORT_FAMILIES)
def test_export_merges_the_deltas(device, tmp_path, family):
    src = write_hf_dir(str(tmp_path / "src"), family)
    with open(os.path.join(src, "tokenizer.json"), "w") as f:
        f.write('{"model": "stand-in"}')
    out = str(tmp_path / "out")
    m = ditch_b200.Model.from_checkpoint(device, src, max_seq=64)
    spec = m.spec
    try:
        edit_model(m, spec)
        shard = 16 << 10 if family == "qwen2" else 0  # several shards for one family
        m.export(out, max_shard_bytes=shard)
        config, dtypes, raw, vals = source_values(family)
        got = read_dir(out)
        assert set(got) == set(vals), (set(got) ^ set(vals))
        n_edited = 0
        for name, (v, own) in vals.items():
            dt, shape, arr = got[name]
            assert dt == own, name
            want, is_edit = expected_values(m, spec, name, v)
            n_edited += is_edit
            if not is_edit and name in raw and dtypes[name] == dt:
                assert arr.tobytes() == raw[name].tobytes(), name  # untouched: the stored bytes
                continue
            want_bits = oracle.f32_to_bf16_bits(want) if dt == "BF16" else (
                oracle.f32_to_f16_bits(want) if dt == "F16" else want)
            assert np.array_equal(arr.reshape(-1), np.asarray(want_bits).reshape(-1)), name
        assert n_edited > 0
        # files
        assert not os.path.exists(os.path.join(out, ".incomplete"))
        assert open(os.path.join(out, "tokenizer.json")).read() == '{"model": "stand-in"}'
        src_cfg = open(os.path.join(src, "config.json")).read()
        quantised = "quantization_config" in config
        want_cfg = ditch_b200.export_config(src_cfg, strip_quantization_config=True) if quantised else src_cfg
        assert open(os.path.join(out, "config.json")).read() == want_cfg
        shards = sorted(f for f in os.listdir(out) if f.endswith(".safetensors"))
        if shard:
            assert len(shards) > 1 and shards[0] == f"model-00001-of-{len(shards):05d}.safetensors"
            index = json.load(open(os.path.join(out, "model.safetensors.index.json")))
            assert set(index["weight_map"]) == set(got)
            assert index["metadata"]["total_size"] == sum(a.nbytes for _, _, a in got.values())
        else:
            assert shards == ["model.safetensors"]
        # the export reloads, and computes what the edited model computes (the
        # merged weights rounded to bf16 against the delta in the epilogue)
        g = Golden(family)
        prompts = g.prompts()
        want_logits = _logits(m, prompts)
        r = ditch_b200.Model.from_checkpoint(device, out, max_seq=64)
        try:
            got_logits = _logits(r, prompts)
        finally:
            r.close()
        err = float(np.abs(got_logits - want_logits).max())
        assert err <= 0.05 * max(1.0, float(np.abs(want_logits).max())), err
    finally:
        m.close()


@pytest.mark.gpu
def test_export_dtype_f32(device, tmp_path):
    """export_dtype f32: every float tensor widened exactly, edited ones merged
    without rounding; config.json names float32."""
    src = write_hf_dir(str(tmp_path / "src"), "qwen2")
    out = str(tmp_path / "out")
    m = ditch_b200.Model.from_checkpoint(device, src, max_seq=64)
    try:
        edit_model(m, m.spec)
        m.export(out, dtype="f32")
        _, _, _, vals = source_values("qwen2")
        got = read_dir(out)
        for name, (v, _) in vals.items():
            dt, _, arr = got[name]
            assert dt == "F32"
            want, _ = expected_values(m, m.spec, name, v)
            assert np.array_equal(arr, want), name
        cfg = json.load(open(os.path.join(out, "config.json")))
        assert cfg["torch_dtype"] == "float32"
    finally:
        m.close()


@pytest.mark.gpu
def test_round_f32(device):
    """The export's rounding against the reference rule (bf16) and IEEE
    round-to-nearest-even (f16, numpy), edges included."""
    rng = np.random.default_rng(0)
    v = np.concatenate([
        rng.standard_normal(4096).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 6, 4096),
        np.array([0.0, -0.0, np.inf, -np.inf, 65504.0, 65519.996, 65520.0, 1e5, 6.1035156e-05, 5.9604645e-08,
                  2.9802322e-08, 2.9802326e-08, 8.940697e-08, 1.0009765625, 1.00048828125, 3.4e38], np.float32),
        (np.arange(1, 2048, dtype=np.float32) * np.float32(2.0 ** -24)),  # the f16 subnormals and their midpoints
        (np.arange(1, 2048, dtype=np.float32) * np.float32(2.0 ** -25)),
    ])
    assert np.array_equal(device.round_f32(v, "bf16"), oracle.f32_to_bf16_bits(v))
    assert np.array_equal(device.round_f32(v, "f16"), oracle.f32_to_f16_bits(v))
    nan = np.array([np.nan, -np.nan], np.float32)
    assert np.isnan(oracle.bf16_bits_to_f32(device.round_f32(nan, "bf16"))).all()
    assert np.array_equal(device.round_f32(nan, "bf16"), oracle.f32_to_bf16_bits(nan))
    assert np.isnan(device.round_f32(nan, "f16").view(np.float16)).all()


@pytest.mark.gpu
def test_export_refuses_gguf(device, tmp_path):
    path = write_gguf_fixture(str(tmp_path / "m.gguf"), "qwen2_gguf")
    m = ditch_b200.Model.from_checkpoint(device, path, max_seq=64)
    try:
        with pytest.raises(ditch_b200.Unsupported, match="GGUF"):
            m.export(str(tmp_path / "out"))
    finally:
        m.close()
