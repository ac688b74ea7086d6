"""Seeded synthetic decoder models (random N(0, 0.02) weights) for parity
tests at head sizes and lengths the reference fixtures do not cover. The same
weights feed the oracle (f32 values of the stored bf16 / FP8 codes) and the
CUDA product (the stored tensors)."""
import numpy as np

import oracle


def make_model(seed, n_layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, inter=512, vocab=300,
               qk_norm=False, qkv_bias=False, fmt="bf16", block=(128, 128), moe=None, eps=1e-6, rope_theta=1e4,
               share_embed_data=False, device_normals=False):
    """share_embed_data: the LM head is given the embedding's values (still
    two tensors, loaded and read separately), which halves the host memory
    of the large-vocabulary shapes. device_normals: the N(0, 1) draws come
    from torch's seeded CUDA generator and are copied to the host (the
    billion-value shapes take minutes with numpy's generator)."""
    from ditch_b200 import Tensor

    rng = np.random.default_rng(seed)
    gen = None
    if device_normals:
        import torch

        gen = torch.Generator(device="cuda").manual_seed(seed)

    def normal(shape):
        if gen is None:
            return rng.standard_normal(shape, dtype=np.float32)
        import torch

        return torch.randn(shape, generator=gen, device="cuda", dtype=torch.float32).cpu().numpy()
    spec = dict(n_layers=n_layers, hidden=hidden, heads=heads, kv_heads=kv_heads, head_dim=head_dim, inter=inter,
                vocab=vocab, eps=eps, rope_theta=rope_theta, qk_norm=int(qk_norm), tied=False)
    if moe:
        spec.update(n_experts=moe["experts"], top_k=moe["top_k"], moe_inter=moe["inter"], norm_topk=1,
                    moe_layers=[True] * n_layers)
    f32, tensors = {}, []

    def bf16(shape, scale=0.02):
        x = normal(shape)
        x *= np.float32(scale)
        bits = oracle.f32_to_bf16_bits(x)
        del x
        return bits, oracle.bf16_bits_to_f32(bits)

    def add(name, rows, cols, quant=False, slabs=None):
        shape = (slabs, rows, cols) if slabs else (rows, cols)
        bits, vals = bf16(shape)
        if quant and fmt == "fp8":
            br, bc = block
            stack_codes, stack_scales, deq = [], [], []
            for w in (vals if slabs else [vals]):
                codes, scales = oracle.quant_fp8_block(w, br, bc)
                stack_codes.append(codes)
                stack_scales.append(scales)
                deq.append(oracle.bf16_bits_to_f32(oracle.dequant_fp8(codes, scales, br, bc)))
            codes = np.stack(stack_codes) if slabs else stack_codes[0]
            scales = np.stack(stack_scales) if slabs else stack_scales[0]
            f32[name] = np.stack(deq) if slabs else deq[0]
            tensors.append(Tensor(name, "fp8", rows, cols, codes, slabs=slabs or 1, scales=scales, block_rows=br,
                                  block_cols=bc))
        elif quant and fmt == "mxfp4":
            blocks, scales, deq = [], [], []
            for w in (vals if slabs else [vals]):
                bl, sc = oracle.quant_mxfp4_packed(w)
                blocks.append(bl)
                scales.append(sc)
                deq.append(oracle.bf16_bits_to_f32(oracle.dequant_mxfp4_packed(bl, sc, rows, cols)))
            f32[name] = np.stack(deq) if slabs else deq[0]
            tensors.append(Tensor(name, "mxfp4", rows, cols, np.stack(blocks) if slabs else blocks[0],
                                  slabs=slabs or 1, scales=np.stack(scales) if slabs else scales[0]))
        else:
            f32[name] = vals
            tensors.append(Tensor(name, "bf16", rows, cols, bits, slabs=slabs or 1))

    def vec(name, n, value=None):
        v = np.full(n, value, np.float32) if value is not None else (1.0 + rng.standard_normal(n) * 0.1).astype(np.float32)
        bits = oracle.f32_to_bf16_bits(v)
        f32[name] = oracle.bf16_bits_to_f32(bits)
        tensors.append(Tensor(name, "bf16", n, 1, bits))

    qd, kvd = heads * head_dim, kv_heads * head_dim
    add("embed", vocab, hidden)
    if share_embed_data:
        f32["lm_head"] = f32["embed"]
        tensors.append(Tensor("lm_head", "bf16", vocab, hidden, tensors[-1].data))
    else:
        add("lm_head", vocab, hidden)
    vec("final_norm", hidden)
    for i in range(n_layers):
        vec(f"L{i}.input_norm", hidden)
        vec(f"L{i}.post_norm", hidden)
        add(f"L{i}.q", qd, hidden, quant=True)
        add(f"L{i}.k", kvd, hidden, quant=True)
        add(f"L{i}.v", kvd, hidden, quant=True)
        add(f"L{i}.o", hidden, qd, quant=True)
        if qkv_bias:
            for nm, n in (("qb", qd), ("kb", kvd), ("vb", kvd)):
                b = (rng.standard_normal(n) * 0.02).astype(np.float32)
                bits = oracle.f32_to_bf16_bits(b)
                f32[f"L{i}.{nm}"] = oracle.bf16_bits_to_f32(bits)
                tensors.append(Tensor(f"L{i}.{nm}", "bf16", n, 1, bits))
        if qk_norm:
            vec(f"L{i}.q_norm", head_dim)
            vec(f"L{i}.k_norm", head_dim)
        if moe:
            add(f"L{i}.router", moe["experts"], hidden)
            add(f"L{i}.e_gate", moe["inter"], hidden, quant=True, slabs=moe["experts"])
            add(f"L{i}.e_up", moe["inter"], hidden, quant=True, slabs=moe["experts"])
            add(f"L{i}.e_down", hidden, moe["inter"], quant=True, slabs=moe["experts"])
        else:
            add(f"L{i}.gate", inter, hidden, quant=True)
            add(f"L{i}.up", inter, hidden, quant=True)
            add(f"L{i}.down", hidden, inter, quant=True)
    return spec, f32, tensors


def prompts(seed, lengths, vocab):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, n).astype(np.uint32) for n in lengths]
