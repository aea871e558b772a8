"""Multi-rank host logic on CPU: two gloo ranks (one process each, like one process per GPU).

What runs across GPUs is the work partition (heads or sequences per rank, no collective on
the data path) and, for the head-sharded varlen prefill, one all-gather of the outputs. Here
each rank computes its share with the CPU oracle and the gathered result must equal the
unsharded computation exactly (heads are independent), the rank-major gather must land
every head where the reference's o_proj reads it, and the step time reported is the maximum
over ranks.
"""
import os
import socket

import numpy as np
import pytest

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, outdir):
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path[:0] = [root, os.path.join(root, "kimi-k3-in-c_b200")]
    import torch.distributed as dist
    import sharding
    import workloads as W
    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60))
    try:
        # head-sharded varlen prefill (config-3 shape class, scaled down)
        rng = np.random.default_rng(5)
        H, d = 4, 16
        cu = np.array([0, 3, 40, 41, 90], np.int32)
        t = W.kda_tokens(rng, int(cu[-1]), H, d, d, bf16=False)
        hs = sharding.head_shard(H, WORLD, rank)
        loc = {k: np.ascontiguousarray(t[k][:, hs]) for k in ("q", "k", "v", "g", "beta")}
        o_loc, _ = oracle.kda_recurrence(loc["q"], loc["k"], loc["v"], loc["g"], loc["beta"], cu)
        o_all = sharding.allgather_heads_host(dist, o_loc)
        np.save(os.path.join(outdir, f"o_{rank}.npy"), o_all)
        # max-over-ranks step time (bench.py reports the slowest rank)
        import torch
        x = torch.tensor([1.0 + rank], dtype=torch.float64)
        dist.all_reduce(x, op=dist.ReduceOp.MAX)
        np.save(os.path.join(outdir, f"max_{rank}.npy"), x.numpy())
        # the NCCL unique id travels as bytes from rank 0
        obj = [b"\x01\x02id-bytes" if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        np.save(os.path.join(outdir, f"uid_{rank}.npy"), np.frombuffer(obj[0], np.uint8))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def two_ranks(tmp_path_factory):
    import multiprocessing as mp
    out = str(tmp_path_factory.mktemp("ranks"))
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, out)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return out


def test_head_sharded_prefill_equals_unsharded(two_ranks):
    import workloads as W
    from oracle import oracle
    rng = np.random.default_rng(5)
    H, d = 4, 16
    cu = np.array([0, 3, 40, 41, 90], np.int32)
    t = W.kda_tokens(rng, int(cu[-1]), H, d, d, bf16=False)
    o_ref, _ = oracle.kda_recurrence(t["q"], t["k"], t["v"], t["g"], t["beta"], cu)
    for r in range(WORLD):
        o = np.load(os.path.join(two_ranks, f"o_{r}.npy"))
        assert o.shape == o_ref.shape
        assert np.array_equal(o, o_ref)


def test_step_time_is_max_over_ranks(two_ranks):
    for r in range(WORLD):
        assert float(np.load(os.path.join(two_ranks, f"max_{r}.npy"))[0]) == float(WORLD)


def test_unique_id_broadcast(two_ranks):
    for r in range(WORLD):
        assert bytes(np.load(os.path.join(two_ranks, f"uid_{r}.npy"))) == b"\x01\x02id-bytes"


def test_gather_layout_and_partitions():
    import sharding
    R, T, hl, dv = 3, 5, 2, 4
    g = np.arange(R * T * hl * dv, dtype=np.float32).reshape(R, T, hl, dv)
    full = sharding.gathered_to_heads(g)
    for r in range(R):
        assert np.array_equal(full[:, r * hl:(r + 1) * hl], g[r])
    assert [sharding.head_shard(64, 8, r) for r in (0, 7)] == [slice(0, 8), slice(56, 64)]
    with pytest.raises(ValueError):
        sharding.head_shard(64, 3, 0)
    sl = [sharding.sequence_shard(10, 4, r) for r in range(4)]
    assert [s.stop - s.start for s in sl] == [3, 3, 2, 2] and sl[-1].stop == 10
