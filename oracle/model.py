"""The oracle forward over a model given as f32 numpy weights.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Weights use canonical names shared with the CUDA product's loader:
``embed``, ``final_norm``, ``lm_head`` and per layer ``L{i}.input_norm``,
``L{i}.post_norm``, ``L{i}.q|k|v|o``, ``L{i}.qb|kb|vb``, ``L{i}.q_norm|k_norm``,
``L{i}.gate|up|down`` (dense) or ``L{i}.router`` + ``L{i}.e_gate|e_up|e_down``
(``[E][..][..]`` stacks, MoE).
"""
import ctypes as C

import numpy as np

from . import Config, Layer, Model, f32, f32p, lib, ptr, szp, u32p


LINEAR = ("q", "k", "v", "o", "gate", "up", "down", "router", "e_gate", "e_up", "e_down")


class OracleModel:
    def __init__(self, spec, weights, weights_bf16=False):
        """weights_bf16: the linear weights and lm_head are given as bf16 bit
        arrays (uint16) and multiplied through ditch's half-precision path, as
        a checkpoint held in bf16 is (mapped mode); the rest stays f32."""
        self.spec = spec
        self.w_bf16 = bool(weights_bf16)

        def keep(k, v):
            linear = k == "lm_head" or k.split(".")[-1] in LINEAR
            if self.w_bf16 and linear:
                return np.ascontiguousarray(v, np.uint16)
            return f32(v)

        self.w = {k: keep(k, v) for k, v in weights.items()}
        self._keep = []
        self.deltas = {}  # (layer, "o"|"down"|("e", e)) -> (a [cols], b [rows])

    def set_delta(self, layer, comp, a, b):
        self.deltas[(layer, comp)] = (f32(a), f32(b))

    def reset_deltas(self):
        self.deltas = {}

    def _build(self):
        s = self.spec
        cfg = Config(
            n_layers=s["n_layers"], hidden=s["hidden"], heads=s["heads"], kv_heads=s["kv_heads"],
            head_dim=s["head_dim"], inter=s["inter"], vocab=s["vocab"], eps=s["eps"],
            rope_theta=s["rope_theta"], qk_norm=int(s.get("qk_norm", 0)),
            rope_scaling=int(s.get("rope_scaling", 0)), rope_factor=s.get("rope_factor", 1.0),
            rope_low_ff=s.get("rope_low_ff", 1.0), rope_high_ff=s.get("rope_high_ff", 1.0),
            rope_orig_max=s.get("rope_orig_max", 1.0), n_experts=s.get("n_experts", 0),
            top_k=s.get("top_k", 0), moe_inter=s.get("moe_inter", 0),
            norm_topk=int(s.get("norm_topk", 1)), rope_attention_factor=s.get("rope_attention_factor", 1.0),
            rope_beta_fast=s.get("rope_beta_fast", 32.0), rope_beta_slow=s.get("rope_beta_slow", 1.0),
            rope_truncate=int(s.get("rope_truncate", 1)))
        layers = (Layer * s["n_layers"])()
        keep = []
        if s.get("rope_factors") is not None:
            rf = np.ascontiguousarray(s["rope_factors"], np.float32)
            keep.append(rf)
            cfg.rope_factors, cfg.n_rope_factors = ptr(rf), rf.size

        def g(name):
            a = self.w.get(name)
            if a is None:
                return None
            return C.cast(a.ctypes.data_as(C.c_void_p), f32p) if a.dtype == np.uint16 else ptr(a)

        for i in range(s["n_layers"]):
            L = layers[i]
            for f in ("input_norm", "post_norm", "q", "k", "v", "o", "qb", "kb", "vb", "q_norm",
                      "k_norm", "gate", "up", "down", "router", "e_gate", "e_up", "e_down"):
                setattr(L, f, g(f"L{i}.{f}"))
            if (i, "o") in self.deltas:  # a [rank][cols] (or [cols]), b [rows][rank] (or [rows])
                a, b = self.deltas[(i, "o")]
                L.o_da, L.o_db, L.o_rank = ptr(a), ptr(b), a.shape[0] if a.ndim == 2 else 1
            if (i, "down") in self.deltas:
                a, b = self.deltas[(i, "down")]
                L.down_da, L.down_db, L.down_rank = ptr(a), ptr(b), a.shape[0] if a.ndim == 2 else 1
            E = s.get("n_experts", 0)
            if E and f"L{i}.router" in self.w:
                da = (f32p * E)()
                db = (f32p * E)()
                dr = (C.c_size_t * E)()
                for e in range(E):
                    if (i, ("e", e)) in self.deltas:
                        a, b = self.deltas[(i, ("e", e))]
                        da[e], db[e] = ptr(a), ptr(b)
                        dr[e] = a.shape[0] if a.ndim == 2 else 1
                L.e_down_da = C.cast(da, C.POINTER(f32p))
                L.e_down_db = C.cast(db, C.POINTER(f32p))
                L.e_down_rank = C.cast(dr, szp)
                keep += [da, db, dr]
        m = Model(c=cfg, embed=g("embed"), final_norm=g("final_norm"), lm_head=g("lm_head"),
                  layers=C.cast(layers, C.POINTER(Layer)), w_bf16=int(self.w_bf16))
        self._keep = [layers, keep]
        return m

    def forward(self, tokens, row_b, row_pos, capture_rows=(), logit_rows=()):
        """Returns (residuals [L+1][nc][H], logits [nl][V])."""
        s = self.spec
        m = self._build()
        tokens = np.ascontiguousarray(tokens, np.uint32)
        rb = np.ascontiguousarray(row_b, np.uint32)
        rp = np.ascontiguousarray(row_pos, np.uint32)
        cap = np.ascontiguousarray(capture_rows, np.uintp)
        lr = np.ascontiguousarray(logit_rows, np.uintp)
        res = np.zeros((s["n_layers"] + 1, len(cap), s["hidden"]), np.float32)
        logits = np.zeros((len(lr), s["vocab"]), np.float32)
        rc = lib().or_forward(C.byref(m), ptr(tokens, u32p), ptr(rb, u32p), ptr(rp, u32p), len(tokens),
                              ptr(cap, szp) if len(cap) else None, len(cap), ptr(res) if len(cap) else None,
                              ptr(lr, szp) if len(lr) else None, len(lr), ptr(logits) if len(lr) else None)
        if rc != 0:
            raise ValueError("oracle forward failed (token id outside the embedding table?)")
        return res, logits


    def generate(self, prompts, max_new_tokens, eos_ids=()):
        """Greedy generation restated from model.generate
        (src/model.zig:5378-5444): the first token from each prompt's last
        logits, then one token per step for every prompt still active; a
        prompt stops after an EOS token (kept) or after max_new_tokens tokens
        (at least one is produced). Each step re-runs the forward over the
        whole sequences: the reference's cached decode step computes the same
        per-query arithmetic over the same keys.

        Returns (tokens, margins): per prompt the token list and, per token,
        the gap between the two largest logits of the row it was picked from
        (a tie-closeness measure for comparisons at float tolerance)."""
        eos = set(int(e) for e in eos_ids)
        seqs = [list(map(int, p)) for p in prompts]
        out = [[] for _ in prompts]
        gaps = [[] for _ in prompts]
        active = list(range(len(prompts)))
        steps = max(int(max_new_tokens), 1)
        for step in range(steps):
            toks, rb, rp, _, _, _, last = flatten_batch([seqs[i] for i in active])
            _, logits = self.forward(toks, rb, rp, logit_rows=last)
            still = []
            for j, i in enumerate(active):
                t, gap = argmax_first(logits[j])
                out[i].append(t)
                gaps[i].append(gap)
                seqs[i].append(t)
                if t not in eos and step + 1 < steps:
                    still.append(i)
            active = still
            if not active:
                break
        return out, gaps


def argmax_first(x):
    """argmax of src/model.zig:5194-5204: a scan from -inf at index 0 with a
    strict `>`, so the first maximum wins and NaN never does. Also returns
    the gap between the two largest values (inf with one candidate)."""
    v = np.where(np.isnan(x), -np.inf, x).astype(np.float64)
    i = int(np.argmax(v))
    if not np.isfinite(v[i]) and v[i] < 0:
        return 0, np.inf
    rest = np.delete(v, i)
    second = rest.max() if rest.size else -np.inf
    return i, float(v[i] - second)


def flatten_batch(prompts, window=1):
    """Flattens prompts into (tokens, row_b, row_pos, capture, first_capture,
    take, last_rows) as src/engine.zig:392-410 does."""
    tokens, rb, rp, capture, first, take, last = [], [], [], [], [], [], []
    idx = 0
    for b, p in enumerate(prompts):
        tk = min(window, len(p))
        first.append(len(capture))
        take.append(tk)
        for pos, t in enumerate(p):
            tokens.append(t)
            rb.append(b)
            rp.append(pos)
            if pos + tk >= len(p):
                capture.append(idx)
            idx += 1
        last.append(idx - 1)
    return (np.array(tokens, np.uint32), np.array(rb, np.uint32), np.array(rp, np.uint32),
            np.array(capture, np.uintp), np.array(first, np.uintp), np.array(take, np.uintp),
            np.array(last, np.uintp))
