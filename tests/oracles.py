"""Plain PyTorch fp32 oracles for the native kernels and the LM engine."""

from __future__ import annotations

import math

import torch


def gelu_tanh(x):
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3)))


def rmsnorm(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def attention(q, k, v, causal, scale):
    """q,k,v [B, T, H, D] fp32 -> [B, T, H, D]."""
    qh, kh, vh = (t.permute(0, 2, 1, 3) for t in (q, k, v))
    s = (qh @ kh.transpose(-1, -2)) * scale
    if causal:
        T = q.shape[1]
        mask = torch.triu(torch.ones(T, T, dtype=torch.bool, device=q.device), 1)
        s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, -1)
    return (p @ vh).permute(0, 2, 1, 3)


def lm_loss(params: dict, ids, targets, spec, causal=True):
    """fp32 TransformerLM loss with the engine's architecture and parameter names."""
    B, T = ids.shape
    F, H = spec.features, spec.heads
    D = F // H
    x = params["token_embedding.weight"][ids] + params["position_embedding.weight"][:T]
    for i in range(spec.layers):
        p = f"blocks.{i}."
        h = rmsnorm(x, params[p + "attn_norm.weight"], spec.eps)

        def lin(t, name):
            y = t @ params[p + name + ".weight"].t()
            b = params.get(p + name + ".bias")
            return y + b if b is not None else y

        q = lin(h, "attn.q_proj").view(B, T, H, D)
        k = lin(h, "attn.k_proj").view(B, T, H, D)
        v = lin(h, "attn.v_proj").view(B, T, H, D)
        o = attention(q, k, v, causal, 1.0 / math.sqrt(D)).reshape(B, T, F)
        x = x + lin(o, "attn.out_proj")
        h2 = rmsnorm(x, params[p + "mlp_norm.weight"], spec.eps)
        x = x + lin(gelu_tanh(lin(h2, "mlp.net.0")), "mlp.net.2")
    hf = rmsnorm(x, params["norm.weight"], spec.eps)
    head = params["token_embedding.weight"] if spec.tied else params["head.weight"]
    logits = hf @ head.t()
    return torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]), targets.reshape(-1))


def rel_err(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-6)).item()
