"""The head-sharded output exchange: k3cuda_allgather_heads (NCCL all-gather over NVLink and
the head interleave) against the host index map of sharding.gathered_to_heads, and
k3cuda_kda_prefill_gathered (the prefill writing every rank's full output over NVLink)
against the unsharded k3cuda_kda_prefill.

One rank on one GPU always runs; two ranks run as two processes when the box has two GPUs
(NCCL takes one GPU per rank). NVLS is switched off for the two-rank run.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

T, HL, DV = 37, 4, 128


def _local_out(rank):
    rng = np.random.default_rng(100 + rank)
    return rng.integers(0, 1 << 16, size=(T, HL, DV), dtype=np.uint16)  # bf16 bit patterns


def _gather(ctx, k3cuda, world, rank, uid):
    ctx.comm_init(world, rank, uid)
    local = ctx.upload(_local_out(rank))
    full = ctx.empty((T, world * HL, DV), np.uint16)
    n = ctx.allgather_heads_workspace(world, T, HL, DV)
    ws = ctx.empty((max(n, 1),), np.uint8)
    for _ in range(2):  # twice: the workspace and communicator are reused
        full.zero()
        ctx.allgather_heads(full, local, T, HL, DV, ws, n)
    return full.numpy()


def test_allgather_single_rank():
    import k3cuda
    import sharding
    c = k3cuda.Context(0)  # its own context: the communicator stays with it
    out = _gather(c, k3cuda, 1, 0, k3cuda.comm_unique_id())
    c.close()
    assert np.array_equal(out, sharding.gathered_to_heads(_local_out(0)[None]))


def _prefill_case(H):
    import workloads as W
    rng = np.random.default_rng(31)
    cu = np.array([0, 70, 71, 200, 330], np.int32)
    t = W.kda_tokens(rng, int(cu[-1]), H, 128, 128, bf16=True)
    return cu, t


def _fused_vs_unsharded(c, k3cuda, world, rank):
    """This rank's head shard through the fused prefill + exchange, and the whole head set
    through k3cuda_kda_prefill on the same GPU; returns (gathered full, unsharded full,
    local state, unsharded state of this rank's heads)."""
    import sharding
    import workloads as W
    H = 2 * world
    cu, t = _prefill_case(H)
    T, n = int(cu[-1]), len(cu) - 1
    hs = sharding.head_shard(H, world, rank)
    Hl = hs.stop - hs.start
    bf = W.f32_to_bf16
    up = lambda x: c.upload(np.ascontiguousarray(x))
    qs = 1.0 / np.sqrt(128.0)
    # fused: local heads, output straight into every rank's full buffer
    full = c.empty((T, H, 128), np.uint16)
    c.comm_register_full(full)
    S = c.upload(np.zeros((n, Hl, 128, 128), np.float32))
    nws = c.kda_prefill_workspace(cu, Hl, 128, 128)
    ws = c.empty((nws,), np.uint8)
    args = [up(bf(t[x][:, hs])) for x in ("q", "k", "v")] + [up(t["g"][:, hs]), up(t["beta"][:, hs])]
    for _ in range(2):
        full.zero()
        S.zero()
        c.kda_prefill_gathered(S, *args, cu, Hl, 128, 128, qs, ws, nws)
    got, got_S = full.numpy(), S.numpy()
    # unsharded reference run of the same kernels
    S2 = c.upload(np.zeros((n, H, 128, 128), np.float32))
    o2 = c.empty((T, H, 128), np.uint16)
    nws2 = c.kda_prefill_workspace(cu, H, 128, 128)
    ws2 = c.empty((nws2,), np.uint8)
    args2 = [up(bf(t[x])) for x in ("q", "k", "v")] + [up(t["g"]), up(t["beta"])]
    c.kda_prefill(S2, o2, *args2, cu, H, 128, 128, qs, ws2, nws2)
    return got, o2.numpy(), got_S, S2.numpy()[:, hs]


def test_prefill_gathered_single_rank():
    """One rank: the fused entry point equals k3cuda_kda_prefill bit for bit."""
    import k3cuda
    c = k3cuda.Context(0)
    c.comm_init(1, 0, k3cuda.comm_unique_id())
    got, want, got_S, want_S = _fused_vs_unsharded(c, k3cuda, 1, 0)
    c.close()
    assert np.array_equal(got, want) and np.array_equal(got_S, want_S)


def _rank_main(rank, world, port, outdir):
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [root, os.path.join(root, "kimi-k3-in-c_b200")]
    import torch.distributed as dist
    import k3cuda
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        obj = [k3cuda.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx = k3cuda.Context(rank)
        out = _gather(ctx, k3cuda, world, rank, obj[0])
        np.save(os.path.join(outdir, f"full_{rank}.npy"), out)
        got, want, got_S, want_S = _fused_vs_unsharded(ctx, k3cuda, world, rank)
        ctx.close()
        np.save(os.path.join(outdir, f"fused_ok_{rank}.npy"),
                np.array([np.array_equal(got, want), np.array_equal(got_S, want_S)]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_allgather_two_ranks(tmp_path):
    import k3cuda
    import sharding
    if k3cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    want = sharding.gathered_to_heads(np.stack([_local_out(r) for r in range(2)]))
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"full_{r}.npy"), want)
        # the fused prefill + exchange equals the unsharded prefill on every rank
        assert np.load(tmp_path / f"fused_ok_{r}.npy").all(), r
