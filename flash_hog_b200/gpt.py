"""Gradient-norm-penalty training step on a pre-LN GPT, attention on the sm_100a kernels.

The benchmarked workload is a random-init 12-layer pre-LN GPT (d_model 768, 12 heads
of 64, causal, MLP 3072, vocab 32000, sequence 1024, 4 sequences per GPU) trained on
the objective

    L_total = L + lam * || dL/dtheta ||^2

whose gradient needs the double backward of every layer. Attention's double
backward runs on this package's kernels through ``dot_product_attention`` (two
nested autograd Functions, the analogue of the reference's nested custom_vjp).
With ``fused=True`` (the default for the "flash" model) LayerNorm, the MLP's GELU
and the cross-entropy loss run on the fused kernels of ``flash_hog_b200.fused`` --
forward, backward and double backward one kernel each -- and the MLP's contractions
on cuBLAS (plain GEMMs); the embeddings stay in torch autograd. Data
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

from flash_hog_b200 import _capi
from flash_hog_b200 import fused as fused_ops
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
    def __init__(self, cfg: GPTConfig, attention, fused: bool):
        super().__init__()
        ln = fused_ops.LayerNorm if fused else nn.LayerNorm
        self.cfg, self.attention = cfg, attention
        self.act = fused_ops.gelu if fused else F.gelu
        self.ln1 = ln(cfg.d_model)
        self.qkv = nn.Linear(cfg.d_model, 3 * cfg.d_model)
        self.proj = nn.Linear(cfg.d_model, cfg.d_model)
        self.ln2 = ln(cfg.d_model)
        self.fc1 = nn.Linear(cfg.d_model, cfg.d_mlp)
        self.fc2 = nn.Linear(cfg.d_mlp, cfg.d_model)

    def forward(self, x):
        b, t, d = x.shape
        h = self.cfg.n_head
        # One projection, then one copy to (3, b, t, h, dh): q, k and v come out contiguous,
        # so the attention op (and its backward and double backward) copies none of them.
        qkv = self.qkv(self.ln1(x)).view(b, t, 3, h, d // h).permute(2, 0, 1, 3, 4).contiguous()
        q, k, v = qkv.unbind(0)
        x = x + self.proj(self.attention(q, k, v, is_causal=True).reshape(b, t, d))
        return x + self.fc2(self.act(self.fc1(self.ln2(x))))


class GPT(nn.Module):
    """Pre-LN GPT; ``attention`` is "flash" (the sm_100a op) or "naive" (torch math);
    ``fused`` (default: with "flash") puts LayerNorm and GELU on the fused kernels."""

    def __init__(self, cfg: GPTConfig, attention: str = "flash", fused: bool | None = None):
        super().__init__()
        fn = {"flash": dot_product_attention, "naive": naive_attention}[attention]
        fused = attention == "flash" if fused is None else fused
        self.cfg, self.fused = cfg, fused
        self.wte = nn.Embedding(cfg.vocab, cfg.d_model)
        self.wpe = nn.Embedding(cfg.seq_len, cfg.d_model)
        self.blocks = nn.ModuleList(Block(cfg, fn, fused) for _ in range(cfg.n_layer))
        self.ln_f = (fused_ops.LayerNorm if fused else nn.LayerNorm)(cfg.d_model)
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
    if getattr(model, "fused", False):  # one kernel per pass, gradient in the logits' dtype
        loss = fused_ops.cross_entropy(logits.flatten(0, 1), tokens[:, 1:].flatten())
    else:
        loss = F.cross_entropy(logits.float().flatten(0, 1), tokens[:, 1:].flatten())
    params = [p for p in model.parameters() if p.requires_grad]
    grads = torch.autograd.grad(loss, params, create_graph=True)
    if getattr(model, "fused", False):  # multi-tensor kernels instead of three per parameter
        penalty = fused_ops.sum_of_squares(grads)
    else:
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


class PenaltyStepGraph:
    """The compute of one grad-norm-penalty step -- forward, ``autograd.grad`` with
    ``create_graph``, the penalty and ``backward()`` into the parameters' ``.grad`` --
    captured once as a CUDA graph and replayed for each new token batch.

    The step launches thousands of small kernels (every layer differentiated twice),
    so launched one by one from Python it is bound by host launch latency; replayed
    as one graph it runs at the GPU's pace. Shapes, parameters and ``.grad`` tensors
    stay fixed (the graph writes the gradients in place: do not reset them with
    ``zero_grad(set_to_none=True)`` between replays); the data-parallel gradient
    all-reduce and the optimizer update run after the replay, outside the graph.
    With ``flat_grads`` (default: when a multi-rank process group is initialised) every
    ``.grad`` is a view of one flat fp32 buffer, which the graph zeroes first and the
    backward accumulates into, so the all-reduce runs on it in place (no gather or
    scatter copies); on one GPU the backward's own gradient tensors are kept instead
    (no zeroing, no accumulation pass). Autocast runs with its cast cache off, as graph
    capture requires.
    """

    def __init__(self, model: GPT, batch: int, lam: float, autocast: bool = True, warmup: int = 3,
                 flat_grads: bool | None = None):
        dev = next(model.parameters()).device
        self.model, self.lam, self.autocast = model, lam, autocast
        self.tokens = torch.zeros((batch, model.cfg.seq_len + 1), dtype=torch.long, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # warm-up off the capture stream (allocator and library set-up)
            for _ in range(warmup):
                model.zero_grad(set_to_none=True)
                self._compute()
        torch.cuda.current_stream(dev).wait_stream(side)
        if flat_grads is None:
            import torch.distributed as dist

            flat_grads = dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1
        self.flat = None
        model.zero_grad(set_to_none=True)
        if flat_grads:
            params = [p for p in model.parameters() if p.requires_grad]
            if any(p.dtype != torch.float32 for p in params):
                raise ValueError("flat_grads keeps the gradients in one fp32 buffer: fp32 parameters only")
            self.flat = torch.zeros(sum(p.numel() for p in params), dtype=torch.float32, device=dev)
            off = 0
            for p in params:
                p.grad = self.flat[off:off + p.numel()].view_as(p)
                off += p.numel()
        self.graph = torch.cuda.CUDAGraph()
        n0 = _capi.launch_count()
        # thread_local: calls from other threads (NCCL's watchdog under torchrun) cannot
        # invalidate the capture.
        with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            self.loss, self.penalty = self._compute()
        self.kernels_per_step = _capi.launch_count() - n0  # this library's kernels in one replay

    def _compute(self):
        if getattr(self, "flat", None) is not None:
            self.flat.zero_()  # the backward accumulates into the flat gradient views
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16, enabled=self.autocast, cache_enabled=False):
            total, loss, penalty = penalty_objective(self.model, self.tokens, self.lam)
        total.backward()
        return loss, penalty

    def step(self, tokens: torch.Tensor, optimizer=None, distributed: bool = False):
        """Copies ``tokens`` into the graph's input, replays the step, then averages the
        gradients over the ranks (``distributed``) and applies ``optimizer``. Returns the
        (loss, penalty) device scalars, overwritten by the next replay."""
        self.tokens.copy_(tokens, non_blocking=True)
        self.graph.replay()
        if distributed and self.flat is not None:
            import torch.distributed as dist

            dist.all_reduce(self.flat)
            self.flat /= dist.get_world_size()
        elif distributed:
            allreduce_grads(self.model)
        if optimizer is not None:
            optimizer.step()
        return self.loss, self.penalty


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
