"""Multi-process host logic on CPU (gloo, world size 2).

* Sharding: each rank runs the double backward (CPU oracle standing in for the
  kernels) on its batch x heads slice; the gathered slices equal the unsharded
  result exactly -- no data-path collective is needed.
* Failure detection without a GPU: a rank that dies before a collective makes
  the survivor's next collective fail within the process-group timeout instead
  of hanging.
"""

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _shard_worker(rank, world, port, outdir):
    _init(rank, world, port, 60)
    from flash_hog_b200.sharding import BatchHeadsSharding
    from oracle import attention_oracle as ora

    x = ora.make_inputs(2, 4, 64, 64, 64, seed=3, dtype=torch.float64)
    o, lse = ora.attention_fwd(x["q"].numpy(), x["k"].numpy(), x["v"].numpy(), causal=True)
    sh = BatchHeadsSharding(2, 4, world)
    pick = lambda t: np.ascontiguousarray(sh.shard(t, rank))
    outs = ora.bwdbwd_stats(pick(x["q"].numpy()), pick(x["k"].numpy()), pick(x["v"].numpy()), pick(o),
                            np.ascontiguousarray(sh.shard_stats(lse, rank)), pick(x["do"].numpy()),
                            pick(x["ddq"].numpy()), pick(x["ddk"].numpy()), pick(x["ddv"].numpy()), causal=True)
    gathered = []
    for t in outs:
        buf = [torch.empty_like(torch.from_numpy(t)) for _ in range(world)]
        dist.all_gather(buf, torch.from_numpy(t))
        gathered.append([b.numpy() for b in buf])
    if rank == 0:
        full = ora.bwdbwd_stats(x["q"].numpy(), x["k"].numpy(), x["v"].numpy(), o, lse, x["do"].numpy(),
                                x["ddq"].numpy(), x["ddk"].numpy(), x["ddv"].numpy(), causal=True)
        ok = True
        for parts, ref in zip(gathered, full):
            for r, part in enumerate(parts):
                sb, shh = sh.slices(r)
                ok &= bool(np.array_equal(ref[sb, :, shh], part))
        with open(os.path.join(outdir, "result"), "w") as f:
            f.write("ok" if ok else "mismatch")
    dist.destroy_process_group()


def _dying_worker(rank, world, port, outdir):
    _init(rank, world, port, 5)
    t = torch.ones(4)
    dist.all_reduce(t)  # both ranks alive: completes
    if rank == 1:
        os._exit(0)  # leaves between steps, with no collective in flight
    try:
        dist.all_reduce(t)
        status = "no error"
    except Exception as e:  # gloo reports the lost peer / timeout
        status = "detected: " + type(e).__name__
    with open(os.path.join(outdir, "result"), "w") as f:
        f.write(status)
    os._exit(0)


def test_batch_heads_sharding_is_exact(tmp_path):
    ctx = mp.start_processes(_shard_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    while not ctx.join(timeout=120):
        pass
    assert (tmp_path / "result").read_text() == "ok"


def test_lost_rank_is_detected_not_hung(tmp_path):
    ctx = mp.start_processes(_dying_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    try:
        while not ctx.join(timeout=60):
            pass
    except mp.ProcessExitedException:
        pass
    assert (tmp_path / "result").read_text().startswith("detected")


def test_sharding_rule():
    from flash_hog_b200.sharding import BatchHeadsSharding

    s = BatchHeadsSharding(4, 16, 8)
    assert (s.batch_parts, s.head_parts) == (4, 2)
    owned = set()
    for r in range(8):
        sb, sh = s.slices(r)
        owned |= {(b, h) for b in range(sb.start, sb.stop) for h in range(sh.start, sh.stop)}
    assert owned == {(b, h) for b in range(4) for h in range(16)}
    with pytest.raises(ValueError):
        BatchHeadsSharding(1, 3, 2)


def _oracle_device(Q, K, V, O, dO, ddQ, ddK, ddV, L, causal, window, scale, policy=None, packed=None):
    """CPU stand-in for the kernels inside flash_bwdbwd (the oracle's explicit formulas)."""
    from oracle import attention_oracle as ora

    b, t, n, _ = Q.shape
    np_ = lambda x: x.detach().double().numpy()
    outs, stats = ora.bwdbwd_stats(*(np_(x) for x in (Q, K, V, O)), L.reshape(b, n, t).double().numpy(),
                                   *(np_(x) for x in (dO, ddQ, ddK, ddV)), scale=scale, causal=causal, window=window,
                                   return_stats=True)
    return tuple(torch.from_numpy(x).to(Q.dtype) for x in outs) + (torch.from_numpy(np.stack(stats)).float(),)


def _sharded_entry_worker(rank, world, port, outdir):
    """sharded_flash_bwdbwd under a real process group (gloo, world 2), grouped-query
    heads, gather=True: every rank ends with the global result of the unsharded call."""
    _init(rank, world, port, 60)
    from flash_hog_b200 import MaskType
    from flash_hog_b200 import bwdbwd as bb
    from flash_hog_b200.sharding import sharded_flash_bwdbwd
    from oracle import attention_oracle as ora

    bb._bwdbwd_device = _oracle_device  # the kernels need a GPU; the host logic is what is tested
    x = ora.make_inputs(2, 4, 48, 64, 32, seed=5, dtype=torch.float64, kv_heads=2)
    o, lse = ora.attention_fwd(x["q"].numpy(), x["k"].numpy(), x["v"].numpy(), causal=2)
    args = [x["q"], x["k"], x["v"], torch.from_numpy(o), x["do"], x["ddq"], x["ddk"], x["ddv"],
            torch.from_numpy(lse)]
    got, sh = sharded_flash_bwdbwd(*args, mask_type=MaskType.CAUSAL_BOTTOM_RIGHT, device="cpu", gather=True)
    want = ora.bwdbwd_stats(*(a.numpy() for a in args[:4]), lse, *(a.numpy() for a in args[4:8]), causal=2)
    ok = sh.world == world and all(np.array_equal(g.numpy(), w_) for g, w_ in zip(got, (want[0], want[1], want[2],
                                                                                       want[3])))
    with open(os.path.join(outdir, f"result{rank}"), "w") as f:
        f.write("ok" if ok else "mismatch")
    dist.destroy_process_group()


def test_sharded_entry_gathers_the_global_result(tmp_path):
    ctx = mp.start_processes(_sharded_entry_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    while not ctx.join(timeout=120):
        pass
    assert (tmp_path / "result0").read_text() == "ok"
    assert (tmp_path / "result1").read_text() == "ok"


def test_sharding_rule_keeps_query_groups_whole():
    from flash_hog_b200.sharding import BatchHeadsSharding

    s = BatchHeadsSharding(1, 8, 4, kv_heads=4)  # groups of 2 query heads
    for r in range(4):
        _, hs = s.slices(r)
        ks = s.kv_slice(r)
        assert {h // 2 for h in range(hs.start, hs.stop)} == set(range(ks.start, ks.stop))
    with pytest.raises(ValueError):
        BatchHeadsSharding(1, 8, 8, kv_heads=4)  # would split a group across ranks
