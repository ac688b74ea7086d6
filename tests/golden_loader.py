"""Loads the committed golden fixtures (tests/golden/<family>.npz) into a
model spec, f32 weights for the oracle and the raw stored tensors for the
CUDA product's loader."""
import json
import os

import numpy as np

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


class Golden:
    def __init__(self, family):
        z = np.load(os.path.join(GOLDEN, family + ".npz"))
        self.family = family
        self.config = json.loads(bytes(z["config_json"]).decode())
        self.dtypes = json.loads(bytes(z["dtypes_json"]).decode())
        self.raw = {k[2:]: z[k] for k in z.files if k.startswith("t/")}
        self.shapes = json.loads(bytes(z["shapes_json"]).decode()) if "shapes_json" in z.files else {}
        self.gguf = bool(self.config.get("gguf"))
        self._canonical_experts()
        self.cases = []
        for i in range(int(z["n_cases"][0])):
            self.cases.append({
                "ids": z[f"case{i}/ids"],
                "last_logits": z[f"case{i}/last_logits"],
                "last_hidden": z[f"case{i}/last_hidden"],
                "argmax": int(z[f"case{i}/argmax"][0]),
            })
        self.spec = self._spec()
        self.block = None
        q = self.config.get("quantization_config")
        if q and q.get("quant_method") == "fp8":
            self.block = tuple(q["weight_block_size"])
        if q and q.get("quant_method") == "compressed-tensors":
            w = q["config_groups"]["group_0"]["weights"]
            self.int_bits, self.int_group = w["num_bits"], w["group_size"]

    def _canonical_experts(self):
        """Routed experts as one tensor per expert and projection, the
        "separate" layout of src/moe.zig:83-92, the host-side step a caller of
        the C ABI performs: mixtral's w1 / w3 / w2 are gate / up / down; the
        fused `experts.gate_up_proj` [E, 2I, hidden] splits into gate rows
        then up rows, and its transposed form [E, hidden, 2I] (with `down_proj`
        [E, I, hidden]) is transposed per expert, as src/moe.zig:728-770."""
        c, raw, dt = self.config, self.raw, self.dtypes
        if c["model_type"] == "mixtral":
            for name in list(raw):
                if ".block_sparse_moe." not in name:
                    continue
                new = name.replace(".block_sparse_moe.", ".mlp.")
                for a, b in ((".w1.", ".gate_proj."), (".w3.", ".up_proj."), (".w2.", ".down_proj.")):
                    new = new.replace(a, b)
                raw[new], dt[new] = raw.pop(name), dt.pop(name)
        H = c["hidden_size"]
        for name in list(raw):
            if not name.endswith(".mlp.experts.gate_up_proj"):
                continue
            p = name[: -len("gate_up_proj")]
            gu, dn = raw.pop(name), raw.pop(p + "down_proj")
            t_gu, t_dn = dt.pop(name), dt.pop(p + "down_proj")
            transposed = gu.shape[1] == H and gu.shape[2] != H
            if transposed:
                gu, dn = np.swapaxes(gu, 1, 2), np.swapaxes(dn, 1, 2)
            inter = gu.shape[1] // 2
            for e in range(gu.shape[0]):
                for proj, arr, t in (("gate_proj", gu[e, :inter], t_gu), ("up_proj", gu[e, inter:], t_gu),
                                     ("down_proj", dn[e], t_dn)):
                    key = f"{p}{e}.{proj}.weight"
                    raw[key], dt[key] = np.ascontiguousarray(arr), t

    def _spec(self):
        c = self.config
        hd = c.get("head_dim") or c["hidden_size"] // c["num_attention_heads"]
        s = dict(n_layers=c["num_hidden_layers"], hidden=c["hidden_size"], heads=c["num_attention_heads"],
                 kv_heads=c["num_key_value_heads"], head_dim=hd, inter=c["intermediate_size"],
                 vocab=c["vocab_size"], eps=c["rms_norm_eps"], rope_theta=c["rope_theta"],
                 qk_norm=int(c["model_type"] in ("qwen3", "qwen3_moe")),
                 tied=bool(c.get("tie_word_embeddings", False)))
        rs = c.get("rope_scaling")
        if rs and rs.get("rope_type") == "llama3":
            s.update(rope_scaling=1, rope_factor=rs["factor"], rope_low_ff=rs["low_freq_factor"],
                     rope_high_ff=rs["high_freq_factor"], rope_orig_max=rs["original_max_position_embeddings"])
        elif self.gguf and "rope_freqs.weight" in self.raw:
            # a GGUF file's per-frequency divisors (src/gguf_model.zig:227-228)
            s.update(rope_scaling=4, rope_factors=np.asarray(self.raw["rope_freqs.weight"], np.float32).ravel())
        if c["model_type"] == "qwen3_moe":
            s.update(n_experts=c["num_experts"], top_k=c["num_experts_per_tok"], moe_inter=c["moe_intermediate_size"],
                     norm_topk=int(c.get("norm_topk_prob", True)))
            mlp_only = set(c.get("mlp_only_layers", []))
            step = c.get("decoder_sparse_step", 1)
            s["moe_layers"] = [(i not in mlp_only) and (i + 1) % step == 0 for i in range(s["n_layers"])]
        if c["model_type"] == "mixtral":  # every layer routed; top-k weights renormalised
            s.update(n_experts=c["num_local_experts"], top_k=c["num_experts_per_tok"], moe_inter=c["intermediate_size"],
                     norm_topk=1, moe_layers=[True] * s["n_layers"])
        return s

    def _heads_permuted(self, name):
        """Heads of a llama.cpp-permuted q / k tensor of a llama GGUF file, else 0."""
        if not (self.gguf and self.config["model_type"] in ("llama", "mistral", "mixtral")):
            return 0
        if name.endswith("attn_q.weight"):
            return self.spec["heads"]
        if name.endswith("attn_k.weight"):
            return self.spec["kv_heads"]
        return 0

    @staticmethod
    def unpermute(a, n_head):
        """llama.cpp's q / k row permutation undone (src/gguf_model.zig:141-143,
        700-800): GGUF row (h, i, half) holds Hugging Face row (h, half, i)."""
        rows = a.shape[0]
        return np.ascontiguousarray(a.reshape(n_head, rows // n_head // 2, 2, -1).swapaxes(1, 2).reshape(a.shape))

    # ---- decoding to f32 (the oracle's view of every weight) ----
    def _dense(self, name):
        """f32 values of a stored weight, decoded like src/dequant.zig does at load."""
        nh = self._heads_permuted(name)
        if nh:
            return self.unpermute(self._dense_raw(name), nh)
        return self._dense_raw(name)

    def _dense_raw(self, name):
        if name in self.raw:
            dt = self.dtypes[name]
            a = self.raw[name]
            if dt == "BF16":
                return oracle.bf16_bits_to_f32(a)
            if dt == "F32":
                return a.astype(np.float32)
            if dt == "F8_E4M3":
                br, bc = self.block
                bits = oracle.dequant_fp8(a, self.raw[name + "_scale_inv"], br, bc)
                return oracle.bf16_bits_to_f32(bits)
            if dt == "F16":
                return a.view(np.float16).astype(np.float32)
            if dt.startswith("GGML_"):  # ggml blocks decoded to f32 as src/quant.zig:57-79
                rows, cols = self.shapes[name]
                code = {"GGML_Q8_0": 5, "GGML_Q4_K": 10, "GGML_Q6_K": 11}[dt]
                return oracle.dequant_ggml(code, a, rows * cols).reshape(rows, cols)
            raise ValueError(f"unsupported dtype {dt} for {name}")
        base = name[: -len(".weight")]
        if base + ".weight_packed" in self.raw:
            rows, cols = (int(v) for v in self.raw[base + ".weight_shape"])
            scales = oracle.bf16_bits_to_f32(self.raw[base + ".weight_scale"])
            zeros = self.raw.get(base + ".weight_zero_point")
            bits = oracle.dequant_int_packed(self.raw[base + ".weight_packed"], scales, zeros, rows, cols,
                                             self.int_bits, self.int_group)
            return oracle.bf16_bits_to_f32(bits)
        raise KeyError(name)

    def hf_names(self):
        """canonical name -> HF tensor name (GGUF names for GGUF fixtures)."""
        s = self.spec
        if self.gguf:
            m = {"embed": "token_embd.weight", "final_norm": "output_norm.weight",
                 "lm_head": "token_embd.weight" if s["tied"] else "output.weight"}
            for i in range(s["n_layers"]):
                p = f"blk.{i}."
                m.update({f"L{i}.input_norm": p + "attn_norm.weight", f"L{i}.post_norm": p + "ffn_norm.weight",
                          f"L{i}.q": p + "attn_q.weight", f"L{i}.k": p + "attn_k.weight",
                          f"L{i}.v": p + "attn_v.weight", f"L{i}.o": p + "attn_output.weight",
                          f"L{i}.qb": p + "attn_q.bias", f"L{i}.kb": p + "attn_k.bias", f"L{i}.vb": p + "attn_v.bias",
                          f"L{i}.gate": p + "ffn_gate.weight", f"L{i}.up": p + "ffn_up.weight",
                          f"L{i}.down": p + "ffn_down.weight"})
            return m
        m = {"embed": "model.embed_tokens.weight", "final_norm": "model.norm.weight",
             "lm_head": "model.embed_tokens.weight" if s["tied"] else "lm_head.weight"}
        for i in range(s["n_layers"]):
            p = f"model.layers.{i}."
            m.update({f"L{i}.input_norm": p + "input_layernorm.weight",
                      f"L{i}.post_norm": p + "post_attention_layernorm.weight"})
            for a, b in (("q", "q_proj"), ("k", "k_proj"), ("v", "v_proj"), ("o", "o_proj")):
                m[f"L{i}.{a}"] = p + f"self_attn.{b}.weight"
            for a, b in (("qb", "q_proj"), ("kb", "k_proj"), ("vb", "v_proj")):
                m[f"L{i}.{a}"] = p + f"self_attn.{b}.bias"
            m[f"L{i}.q_norm"] = p + "self_attn.q_norm.weight"
            m[f"L{i}.k_norm"] = p + "self_attn.k_norm.weight"
            if s.get("moe_layers") and s["moe_layers"][i]:
                m[f"L{i}.router"] = p + "mlp.gate.weight"
            else:
                for a in ("gate", "up", "down"):
                    m[f"L{i}.{a}"] = p + f"mlp.{a}_proj.weight"
        return m

    def has(self, hf):
        base = hf[: -len(".weight")] if hf.endswith(".weight") else hf
        return hf in self.raw or base + ".weight_packed" in self.raw

    def f32_weights(self):
        s = self.spec
        out = {}
        for canon, hf in self.hf_names().items():
            if self.has(hf):
                out[canon] = self._dense(hf)
        if s.get("moe_layers"):
            for i in range(s["n_layers"]):
                if not s["moe_layers"][i]:
                    continue
                p = f"model.layers.{i}.mlp.experts."
                for a in ("gate", "up", "down"):
                    out[f"L{i}.e_{a}"] = np.stack([self._dense(p + f"{e}.{a}_proj.weight")
                                                   for e in range(s["n_experts"])])
        return out

    def prompts(self):
        return [c["ids"].astype(np.uint32) for c in self.cases]

    # ---- the stored tensors, for the CUDA product's loader ----
    def _cuda_tensor(self, canon, hf, slabs=1, stack=None):
        from ditch_b200 import Tensor
        from ditch_b200.cuda import SCALE_BF16, SCALE_F32
        names = stack or [hf]
        first = names[0]
        base = first[: -len(".weight")]
        if first in self.raw:
            dt = self.dtypes[first]
            a = np.stack([self.raw[n] for n in names]) if stack else self.raw[first]
            if not stack and self._heads_permuted(first):
                a = self.unpermute(a, self._heads_permuted(first))
            rows, cols = (a.shape[-2], a.shape[-1]) if a.ndim >= 2 else (a.shape[0], 1)
            if dt == "BF16":
                return Tensor(canon, "bf16", rows, cols, a, slabs=slabs)
            if dt == "F32":
                return Tensor(canon, "f32", rows, cols, a, slabs=slabs)
            if dt == "F8_E4M3":
                br, bc = self.block
                sc = np.stack([self.raw[n + "_scale_inv"] for n in names]) if stack else self.raw[first + "_scale_inv"]
                return Tensor(canon, "fp8", rows, cols, a, slabs=slabs, scales=sc.astype(np.float32),
                              scales_dtype=SCALE_F32, block_rows=br, block_cols=bc)
            if dt == "F16":
                return Tensor(canon, "f16", rows, cols, a, slabs=slabs)
            if dt.startswith("GGML_"):  # raw blocks, as stored
                rows, cols = self.shapes[first]
                return Tensor(canon, {"GGML_Q8_0": "q8_0", "GGML_Q4_K": "q4_k"}[dt], rows, cols, a, slabs=slabs)
            raise ValueError(dt)
        if base + ".weight_packed" in self.raw:
            rows, cols = (int(v) for v in self.raw[base + ".weight_shape"])
            return Tensor(canon, "int", rows, cols, self.raw[base + ".weight_packed"],
                          scales=self.raw[base + ".weight_scale"], scales_dtype=SCALE_BF16,
                          zeros=self.raw.get(base + ".weight_zero_point"), block_cols=self.int_group,
                          bits=self.int_bits)
        raise KeyError(hf)

    def cuda_tensors(self):
        s = self.spec
        out = []
        for canon, hf in self.hf_names().items():
            if self.has(hf):
                out.append(self._cuda_tensor(canon, hf))
        if s.get("moe_layers"):
            for i in range(s["n_layers"]):
                if not s["moe_layers"][i]:
                    continue
                p = f"model.layers.{i}.mlp.experts."
                for a in ("gate", "up", "down"):
                    names = [p + f"{e}.{a}_proj.weight" for e in range(s["n_experts"])]
                    out.append(self._cuda_tensor(f"L{i}.e_{a}", None, slabs=s["n_experts"], stack=names))
        return out
