"""Gradient-norm-penalty training step on a pre-LN GPT, attention on the sm_100a kernels.

The benchmarked workload is a random-init 12-layer pre-LN GPT (d_model 768, 12 heads
of 64, causal, MLP 3072, vocab 32000, sequence 1024, 4 sequences per GPU) trained on
the objective

    L_total = L + lam * || dL/dtheta ||^2

whose gradient needs the double backward of every layer. Attention's double
backward runs on this package's kernels through ``dot_product_attention`` (two
nested autograd Functions, the analogue of the reference's nested custom_vjp);
LayerNorm, the MLP, the embeddings and the loss stay in torch autograd. Data
parallelism: each rank computes the full step on its own token batch and the
parameter gradients (penalty terms included) are averaged with one NCCL
all-reduce over a flat buffer.

The reference repository has no model code; it only differentiates the attention
op twice (flash_hog/jax/attention.py:100-130). The same model with
``attention="naive"`` (torch math attention) is the parity reference in tests.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from flash_hog_b200.attention import dot_product_attention


@dataclass
class GPTConfig:
    n_layer: int = 12
    d_model: int = 768
    n_head: int = 12
    d_mlp: int = 3072
    vocab: int = 32000
    seq_len: int = 1024


def naive_attention(q, k, v, is_causal=True):
    """softmax(q k^T / sqrt(D) + causal mask) v in torch ops (BTNH), for reference runs."""
    scale = q.shape[-1] ** -0.5
    s = torch.einsum("bqhd,bkhd->bhqk", q.float(), k.float()) * scale
    if is_causal:
        keep = torch.ones(q.shape[1], k.shape[1], dtype=torch.bool, device=q.device).tril()
        s = s.masked_fill(~keep, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bhqk,bkhd->bqhd", p, v.float()).to(q.dtype)


class Block(nn.Module):
    def __init__(self, cfg: GPTConfig, attention):
        super().__init__()
        self.cfg, self.attention = cfg, attention
        self.ln1 = nn.LayerNorm(cfg.d_model)
        self.qkv = nn.Linear(cfg.d_model, 3 * cfg.d_model)
        self.proj = nn.Linear(cfg.d_model, cfg.d_model)
        self.ln2 = nn.LayerNorm(cfg.d_model)
        self.fc1 = nn.Linear(cfg.d_model, cfg.d_mlp)
        self.fc2 = nn.Linear(cfg.d_mlp, cfg.d_model)

    def forward(self, x):
        b, t, d = x.shape
        h = self.cfg.n_head
        q, k, v = self.qkv(self.ln1(x)).view(b, t, 3, h, d // h).unbind(2)
        x = x + self.proj(self.attention(q, k, v, is_causal=True).reshape(b, t, d))
        return x + self.fc2(F.gelu(self.fc1(self.ln2(x))))


class GPT(nn.Module):
    """Pre-LN GPT; ``attention`` is "flash" (the sm_100a op) or "naive" (torch math)."""

    def __init__(self, cfg: GPTConfig, attention: str = "flash"):
        super().__init__()
        fn = {"flash": dot_product_attention, "naive": naive_attention}[attention]
        self.cfg = cfg
        self.wte = nn.Embedding(cfg.vocab, cfg.d_model)
        self.wpe = nn.Embedding(cfg.seq_len, cfg.d_model)
        self.blocks = nn.ModuleList(Block(cfg, fn) for _ in range(cfg.n_layer))
        self.ln_f = nn.LayerNorm(cfg.d_model)
        self.apply(self._init)
        for blk in self.blocks:  # GPT-2 style scaled init of the residual projections
            for lin in (blk.proj, blk.fc2):
                nn.init.normal_(lin.weight, std=0.02 / math.sqrt(2 * cfg.n_layer))

    @staticmethod
    def _init(m):
        if isinstance(m, (nn.Linear, nn.Embedding)):
            nn.init.normal_(m.weight, std=0.02)
        if isinstance(m, nn.Linear) and m.bias is not None:
            nn.init.zeros_(m.bias)

    def forward(self, tokens):
        t = tokens.shape[1]
        x = self.wte(tokens) + self.wpe(torch.arange(t, device=tokens.device))
        for blk in self.blocks:
            x = blk(x)
        return self.ln_f(x) @ self.wte.weight.t()  # tied LM head


def penalty_objective(model: GPT, tokens: torch.Tensor, lam: float):
    """(L + lam ||dL/dtheta||^2, L, ||dL/dtheta||^2) for next-token cross-entropy L
    on ``tokens`` (B, T+1); the gradient is kept in the graph (create_graph)."""
    logits = model(tokens[:, :-1])
    loss = F.cross_entropy(logits.float().flatten(0, 1), tokens[:, 1:].flatten())
    params = [p for p in model.parameters() if p.requires_grad]
    grads = torch.autograd.grad(loss, params, create_graph=True)
    penalty = sum((g.float() ** 2).sum() for g in grads)
    return loss + lam * penalty, loss.detach(), penalty.detach()


def allreduce_grads(model: nn.Module, group=None) -> None:
    """Averages parameter gradients over the ranks of ``group``: one all-reduce over
    a flat buffer (NCCL over NVLink on GPUs)."""
    import torch.distributed as dist

    params = [p for p in model.parameters() if p.grad is not None]
    if not params:
        return
    flat = torch.cat([p.grad.reshape(-1) for p in params])
    dist.all_reduce(flat, group=group)
    flat /= dist.get_world_size(group)
    off = 0
    for p in params:
        n = p.grad.numel()
        p.grad.copy_(flat[off:off + n].view_as(p.grad))
        off += n


def train_step(model: GPT, tokens: torch.Tensor, lam: float, optimizer=None, distributed: bool = False,
               autocast: bool = True):
    """One grad-norm-penalty step: objective, its gradient (double backward), the
    data-parallel gradient average and the optimizer update. Returns (loss, penalty)."""
    dev = tokens.device.type
    with torch.autocast(device_type=dev, dtype=torch.bfloat16, enabled=autocast and dev == "cuda"):
        total, loss, penalty = penalty_objective(model, tokens, lam)
    if optimizer is not None:
        optimizer.zero_grad(set_to_none=True)
    total.backward()
    if distributed:
        allreduce_grads(model)
    if optimizer is not None:
        optimizer.step()
    return loss, penalty
