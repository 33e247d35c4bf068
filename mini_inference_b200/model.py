"""A Qwen2 decoder whose attention runs on this package's paged-KV contexts.

This is the caller side of the hot path: the reference's ``Qwen2ForCausalLM``
(``engine/model.py:254-323``) with the same parameters, the same order of
parameters and the same tensor operations for everything around attention (embedding
lookup, RMSNorm with float32 statistics, the fused ``qkv_proj`` with bias, ``o_proj``,
the SwiGLU MLP with the fused ``gate_up_proj``, residual adds, the final norm and the
tied or separate LM head). The projections stay on cuBLAS through PyTorch; the residual
adds, the RMSNorms and the MLP's ``silu(gate) * up`` are this package's kernels, one launch
each (``ops.add_rms_norm``, ``ops.silu_mul``) where the reference runs eager chains of
eight or more. Attention goes through the context the runner passes in:
with this package's contexts the layer hands the raw ``qkv_proj`` output to
``ctx.attend_qkv``, which applies RoPE fused with the KV append (bit-identical to the
reference's ``apply_rope``) and runs the paged attention kernels. A context without
``attend_qkv`` (the reference's own) gets the reference's split, head views, RoPE and
``ctx.attend`` call (``engine/model.py:241-251``).

:func:`init_random` reproduces the weights the task's configurations are quoted on:
``torch.manual_seed(seed)`` and then ``normal_(0, std)`` over the parameters in the
reference model's ``named_parameters()`` order, drawn on the CPU in float32 and cast.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops


@dataclass(frozen=True)
class Qwen2Config:
    """The architecture numbers of ``engine/model.py:37-86`` (same field names)."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position_embeddings: int = 32768
    tie_word_embeddings: bool = True
    attention_bias: bool = True

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    # Shapes of the two model families the task's configurations use.
    @classmethod
    def qwen2_0_5b(cls, **kw) -> "Qwen2Config":
        """Qwen2.5-0.5B: 24 layers, hidden 896, 14 / 2 heads of 64, MLP 4864, vocab 151936, tied head."""
        base = dict(vocab_size=151936, hidden_size=896, intermediate_size=4864, num_layers=24, num_heads=14,
                    num_kv_heads=2, head_dim=64, tie_word_embeddings=True)
        base.update(kw)
        return cls(**base)

    @classmethod
    def qwen2_7b(cls, **kw) -> "Qwen2Config":
        """Qwen2.5-7B: 28 layers, hidden 3584, 28 / 4 heads of 128, MLP 18944, vocab 152064, separate head."""
        base = dict(vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_layers=28, num_heads=28,
                    num_kv_heads=4, head_dim=128, tie_word_embeddings=False, max_position_embeddings=33024)
        base.update(kw)
        return cls(**base)


def parameter_shapes(cfg: Qwen2Config) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) of every parameter in the reference's ``named_parameters()`` order."""
    h, q, kv, inter = cfg.hidden_size, cfg.q_size, cfg.kv_size, cfg.intermediate_size
    out = [("embed_tokens.weight", (cfg.vocab_size, h))]
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        out.append((p + "input_norm.weight", (h,)))
        out.append((p + "attn.qkv_proj.weight", (q + 2 * kv, h)))
        if cfg.attention_bias:
            out.append((p + "attn.qkv_proj.bias", (q + 2 * kv,)))
        out.append((p + "attn.o_proj.weight", (h, q)))
        out.append((p + "post_attn_norm.weight", (h,)))
        out.append((p + "mlp.gate_up_proj.weight", (2 * inter, h)))
        out.append((p + "mlp.down_proj.weight", (h, inter)))
    out.append(("norm.weight", (h,)))
    if not cfg.tie_word_embeddings:
        out.append(("lm_head.weight", (cfg.vocab_size, h)))
    return out


def init_random(cfg: Qwen2Config, seed: int = 0, std: float = 0.02, dtype: torch.dtype = torch.float16,
                device: torch.device | str = "cuda", unit_norms: bool = False,
                generator_device: str = "cpu") -> dict[str, torch.Tensor]:
    """Random weights: ``manual_seed(seed)``, then ``normal_(0, std)`` per parameter in order.

    With ``generator_device="cpu"`` (the default) the draws are the reference's: the
    global CPU generator in float32, parameter by parameter, so a reference model seeded
    the same way holds the same values. ``unit_norms`` then sets every RMSNorm weight to
    1 (its draw is still made, so the other parameters do not change): the norms' own
    initial value, which keeps a random model's tokens dependent on its context.
    ``generator_device="cuda"`` draws on the GPU instead (fast, for benchmarks whose
    weights only need the right shapes and scale).
    """
    params: dict[str, torch.Tensor] = {}
    if generator_device == "cpu":
        torch.manual_seed(seed)
        gen = None
    else:
        gen = torch.Generator(device=device).manual_seed(seed)
    for name, shape in parameter_shapes(cfg):
        if gen is None:
            t = torch.empty(shape, dtype=torch.float32)
            t.normal_(0.0, std)
        else:
            t = torch.empty(shape, dtype=torch.float32, device=device)
            t.normal_(0.0, std, generator=gen)
        if unit_norms and name.endswith("norm.weight"):
            t.fill_(1.0)
        params[name] = t.to(device=device, dtype=dtype)
    return params


def _split_k(rows: int, weight: torch.Tensor) -> int:
    """How many K slices a decode batch's projection by ``weight`` gets (0: one cuBLAS GEMM).

    A long-K, small-N projection of a few rows (down_proj of the 0.5B shape: K = 4864, N =
    896) runs as cuBLAS's single GEMM on few SMs (8.2-8.4 us at 64-256 rows, measured); cut
    into 4-8 slices of one batched GEMM with float32 partials it takes 3.9-5.1 us, and the
    next norm sums the partials. Large weights (the 7B shape) stay whole: they stream HBM.
    """
    n, k = weight.shape
    if rows > 256 or k < 4 * n or weight.numel() * weight.element_size() > (32 << 20):
        return 0
    s = 8 if rows <= 128 else 4
    return s if k % s == 0 else 0


def _linear_split_k(x: torch.Tensor, weight: torch.Tensor, splits: int) -> torch.Tensor:
    """``F.linear(x, weight)`` as float32 partial sums ``[splits, rows, N]`` of one batched cuBLAS GEMM.

    ``ops.add_rms_norm`` takes them as its ``x``: it adds the slices in order and rounds to
    the model dtype, where ``F.linear`` rounds its output.
    """
    rows, k = x.numel() // x.shape[-1], x.shape[-1]
    n = weight.shape[0]
    xs = x.reshape(rows, splits, k // splits).transpose(0, 1)  # [S, rows, K/S]
    ws = weight.view(n, splits, k // splits).permute(1, 2, 0)  # [S, K/S, N]
    return torch.bmm(xs, ws, out_dtype=torch.float32)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat([-x2, x1], dim=-1)


class Qwen2Model:
    """``Qwen2ForCausalLM`` over a dict of weight tensors; ``forward(ids, positions, ctx)`` -> hidden states.

    The call surface is the reference's: ``model(input_ids [B, T], positions [B, T], ctx)``
    returns the final-norm hidden states ``[B, T, hidden]``, ``compute_logits`` applies the
    LM head, ``lm_head_weight`` is the matrix it uses (the embedding when tied) and ``cfg``
    the architecture.
    """

    def __init__(self, cfg: Qwen2Config, weights: dict[str, torch.Tensor]) -> None:
        self.cfg = cfg
        self.w = weights
        self.embed = weights["embed_tokens.weight"]
        self.dtype = self.embed.dtype
        self.device = self.embed.device
        self.lm_head_weight = self.embed if cfg.tie_word_embeddings else weights["lm_head.weight"]
        self.layers = []
        for i in range(cfg.num_layers):
            p = f"layers.{i}."
            self.layers.append((weights[p + "input_norm.weight"], weights[p + "attn.qkv_proj.weight"],
                                weights.get(p + "attn.qkv_proj.bias"), weights[p + "attn.o_proj.weight"],
                                weights[p + "post_attn_norm.weight"], weights[p + "mlp.gate_up_proj.weight"],
                                weights[p + "mlp.down_proj.weight"]))
        self.norm = weights["norm.weight"]
        # The reference's RoPE tables (float32, cast to the model dtype per lookup), built once.
        self.cos, self.sin = ops.rope_tables(cfg.head_dim, cfg.max_position_embeddings, cfg.rope_theta, self.dtype,
                                             self.device)

    def weight_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.w.values())

    def _attention(self, layer: int, x: torch.Tensor, positions: torch.Tensor, ctx, wqkv, bqkv, wo) -> torch.Tensor:
        cfg = self.cfg
        b, t, _ = x.shape
        qkv = F.linear(x, wqkv, bqkv)
        if hasattr(ctx, "attend_qkv"):
            out = ctx.attend_qkv(layer, qkv, self.cos, self.sin, cfg.num_heads)  # [B, Hq, T, d]
        else:  # engine/model.py:241-250 for a context that only has attend()
            q, k, v = qkv.split([cfg.q_size, cfg.kv_size, cfg.kv_size], dim=-1)
            q = q.view(b, t, cfg.num_heads, cfg.head_dim).transpose(1, 2)
            k = k.view(b, t, cfg.num_kv_heads, cfg.head_dim).transpose(1, 2)
            v = v.view(b, t, cfg.num_kv_heads, cfg.head_dim).transpose(1, 2)
            cos, sin = self.cos[positions].unsqueeze(1), self.sin[positions].unsqueeze(1)
            q, k = q * cos + _rotate_half(q) * sin, k * cos + _rotate_half(k) * sin
            out = ctx.attend(layer, q, k, v)
        return F.linear(out.transpose(1, 2).reshape(b, t, cfg.q_size), wo)

    def __call__(self, input_ids: torch.Tensor, positions: torch.Tensor, ctx) -> torch.Tensor:
        return self.forward(input_ids, positions, ctx)

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, ctx) -> torch.Tensor:
        """engine/model.py:266-318: ``x = x + attn(norm(x)); x = x + mlp(norm(x))`` per layer, then the norm.

        ``h`` is the residual stream ``x``; each block's output ``y`` is added into it by the
        next norm's launch (``ops.add_rms_norm``, the reference's rounding), and the MLP's
        ``silu(gate) * up`` is one launch (``ops.silu_mul``). For decode batches of the 0.5B
        shape ``down_proj`` leaves float32 split-K partials that the next norm sums and rounds
        (see :func:`_split_k`).
        """
        eps = self.cfg.rms_norm_eps
        h = F.embedding(input_ids, self.embed)  # a fresh tensor: updated in place below
        y = None
        rows = h.numel() // h.shape[-1]
        splits = _split_k(rows, self.layers[0][6]) if self.layers else 0
        for i, (n1, wqkv, bqkv, wo, n2, wgu, wd) in enumerate(self.layers):
            x = ops.add_rms_norm(h, n1, eps) if y is None else ops.add_rms_norm(y, n1, eps, residual=h)
            y = self._attention(i, x.view_as(h), positions, ctx, wqkv, bqkv, wo)
            x = ops.add_rms_norm(y, n2, eps, residual=h)
            act = ops.silu_mul(F.linear(x, wgu))
            # down_proj: float32 split-K partials for decode batches, summed by the next norm
            y = _linear_split_k(act, wd, splits) if splits else F.linear(act, wd)
        return ops.add_rms_norm(y, self.norm, eps, residual=h).view_as(h)

    def compute_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return F.linear(hidden, self.lm_head_weight)
