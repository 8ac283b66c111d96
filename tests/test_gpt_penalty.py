"""Grad-norm-penalty GPT step: the model with the sm_100a attention op against the
same model with torch math attention, and the data-parallel gradient average.

The penalty L + lam ||dL/dtheta||^2 differentiates every layer twice, so the step
exercises fwd -> bwd -> bwdbwd of the attention op inside a model.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from flash_hog_b200.gpt import GPT, GPTConfig, allreduce_grads, penalty_objective, train_step

SMALL = GPTConfig(n_layer=2, d_model=128, n_head=2, d_mlp=256, vocab=512, seq_len=128)


def _tokens(cfg, batch, seed, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, cfg.vocab, (batch, cfg.seq_len + 1), generator=g).to(device)


@pytest.mark.gpu
def test_penalty_step_matches_math_attention():
    """fp32 model, attention on the kernels (bf16 inside) vs torch math attention:
    loss, penalty and every parameter gradient of L + lam ||dL/dtheta||^2."""
    torch.manual_seed(0)
    ref = GPT(SMALL, attention="naive").cuda()
    ours = GPT(SMALL, attention="flash").cuda()
    ours.load_state_dict(ref.state_dict())
    tokens = _tokens(SMALL, 2, seed=1, device="cuda")
    lam = 0.5
    out = []
    for model in (ref, ours):
        loss, pen = train_step(model, tokens, lam, autocast=False)
        out.append((loss.item(), pen.item(), [p.grad.detach().float().clone() for p in model.parameters()]))
    (l0, p0, g0), (l1, p1, g1) = out
    assert abs(l1 - l0) <= 1e-3 * abs(l0)
    assert abs(p1 - p0) <= 2e-2 * abs(p0)
    num = sum(((a - b) ** 2).sum() for a, b in zip(g1, g0)).sqrt()
    den = sum((b ** 2).sum() for b in g0).sqrt()
    assert (num / den).item() <= 2e-2
    for a, b in zip(g1, g0):
        assert ((a - b).norm() / b.norm().clamp_min(1e-12)).item() <= 5e-2


@pytest.mark.gpu
def test_penalty_step_bf16_autocast_runs():
    """The benchmark's dtype policy (bf16 autocast): finite loss, penalty and gradients."""
    torch.manual_seed(0)
    model = GPT(SMALL, attention="flash").cuda()
    opt = torch.optim.SGD(model.parameters(), lr=1e-3)
    loss, pen = train_step(model, _tokens(SMALL, 2, seed=2, device="cuda"), 0.1, optimizer=opt)
    assert torch.isfinite(loss) and torch.isfinite(pen) and pen.item() > 0
    assert all(torch.isfinite(p).all() for p in model.parameters())


@pytest.mark.gpu
def test_fused_layernorm_gelu_match_torch_modules_in_the_step():
    """fp32 model: LayerNorm and GELU on the fused kernels (forward, backward, double
    backward) against torch's modules, same weights, attention on the kernels in both."""
    from flash_hog_b200.gpt import GPT

    torch.manual_seed(0)
    ref = GPT(SMALL, attention="flash", fused=False).cuda()
    ours = GPT(SMALL, attention="flash", fused=True).cuda()
    ours.load_state_dict(ref.state_dict())
    tokens = _tokens(SMALL, 2, seed=4, device="cuda")
    out = []
    for model in (ref, ours):
        loss, pen = train_step(model, tokens, 0.5, autocast=False)
        out.append((loss.item(), pen.item(), [p.grad.detach().clone() for p in model.parameters()]))
    (l0, p0, g0), (l1, p1, g1) = out
    assert abs(l1 - l0) <= 1e-5 * abs(l0) and abs(p1 - p0) <= 1e-4 * abs(p0)
    for a, b in zip(g1, g0):
        assert ((a - b).norm() / b.norm().clamp_min(1e-12)).item() <= 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("flat_grads", [False, True])
def test_graphed_step_equals_eager_step(flat_grads):
    """The step captured as a CUDA graph and replayed on new tokens gives the eager
    step's loss, penalty and gradients (bf16 autocast, the benchmark's policy), with the
    backward's own gradient tensors and with all gradients in one flat buffer (the
    multi-rank layout, whose buffer the graph zeroes and accumulates into)."""
    from flash_hog_b200.gpt import GPT, PenaltyStepGraph

    torch.manual_seed(0)
    eager = GPT(SMALL, attention="flash").cuda()
    graphed = GPT(SMALL, attention="flash").cuda()
    graphed.load_state_dict(eager.state_dict())
    step = PenaltyStepGraph(graphed, batch=2, lam=0.1, flat_grads=flat_grads)
    assert (step.flat is not None) == flat_grads
    for seed in (21, 22):
        tokens = _tokens(SMALL, 2, seed=seed, device="cuda")
        eager.zero_grad(set_to_none=True)
        l0, p0 = train_step(eager, tokens, 0.1)
        l1, p1 = step.step(tokens)
        torch.cuda.synchronize()
        assert abs(l1.item() - l0.item()) <= 1e-6 * abs(l0.item())
        assert abs(p1.item() - p0.item()) <= 1e-4 * abs(p0.item())
        for a, b in zip(graphed.parameters(), eager.parameters()):
            assert ((a.grad - b.grad).norm() / b.grad.norm().clamp_min(1e-12)).item() <= 1e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        model = GPT(SMALL, attention="naive")
        tokens = _tokens(SMALL, 2, seed=10 + rank)
        train_step(model, tokens, 0.5, distributed=True, autocast=False)
        q.put((rank, [p.grad.numpy().copy() for p in model.parameters()]))  # by value, not shared memory
    finally:
        dist.destroy_process_group()


def test_data_parallel_gradient_average_gloo():
    """world_size 2 on CPU (gloo): every rank ends with the mean of the two ranks'
    penalty-objective gradients, as a single process computes them."""
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expected = None
    for r in range(world):
        torch.manual_seed(0)
        model = GPT(SMALL, attention="naive")
        total, _, _ = penalty_objective(model, _tokens(SMALL, 2, seed=10 + r), 0.5)
        total.backward()
        g = [p.grad.clone() for p in model.parameters()]
        expected = g if expected is None else [a + b for a, b in zip(expected, g)]
    expected = [e / world for e in expected]
    for r in range(world):
        for a, b in zip(got[r], expected):
            assert torch.allclose(torch.from_numpy(a), b, rtol=1e-4, atol=1e-6)
