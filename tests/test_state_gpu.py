"""The state file for device-resident state (k3g_state_save / k3g_state_load): a round
trip restores the device buffers bit for bit, and every refusal of the reference's loader
(src/cli/k3_state.c:102-183) holds: another architecture, another geometry, a cache too
small, a truncated file, a longer file, one damaged byte. The header keeps the reference's
K3StateHdr layout (src/cli/k3_state.h:37-50) under version 4."""
import ctypes as C
import os

import numpy as np
import pytest

import k3cuda

pytestmark = pytest.mark.gpu

FP = np.arange(12, dtype=np.int32) * 7 + 1
HDR = np.dtype([("magic", "S4"), ("version", "<i4"), ("fp", "<i4", 12), ("n_bound", "<i4"),
                ("n_mla", "<i4"), ("cached", "<i4"), ("nseq", "<i4"), ("kper", "<i8"),
                ("kvpp", "<i8"), ("ropepp", "<i8"), ("payload_hash", "<u8")])
IP = C.POINTER(C.c_int)


def _ip(a):
    return a.ctypes.data_as(IP)


@pytest.fixture
def state(ctx, tmp_path):
    G = k3cuda.gpu_lib()
    rng = np.random.default_rng(3)
    n_bound, kper, n_mla, cap, cached = 3, 1000, 2, 50, 37
    ks = rng.standard_normal((n_bound, kper)).astype(np.float32)
    lat = rng.integers(0, 1 << 16, (n_mla, cap, 512), dtype=np.uint16)
    rope = rng.integers(0, 1 << 16, (n_mla, cap, 64), dtype=np.uint16)
    seq = rng.integers(0, 163840, 45, dtype=np.int32)
    d = dict(ks=ctx.upload(ks), lat=ctx.upload(lat), rope=ctx.upload(rope))
    path = str(tmp_path / "s.k3state")
    rc = G.k3g_state_save(path.encode(), _ip(FP), _ip(seq), len(seq), d["ks"].ptr, kper, n_bound,
                          d["lat"].ptr, d["rope"].ptr, n_mla, cap, 512, 64, cached)
    assert rc == 0
    return G, path, dict(ks=ks, lat=lat, rope=rope, seq=seq, n_bound=n_bound, kper=kper,
                         n_mla=n_mla, cap=cap, cached=cached)


def _load(ctx, G, path, s, fp=FP, cap=None, kper=None):
    cap = s["cap"] if cap is None else cap
    kper = s["kper"] if kper is None else kper
    dks = ctx.empty((s["n_bound"], kper), np.float32)
    dlat = ctx.empty((s["n_mla"], cap, 512), np.uint16)
    drope = ctx.empty((s["n_mla"], cap, 64), np.uint16)
    for b in (dks, dlat, drope):
        b.zero()
    seq = np.zeros(100, np.int32)
    nseq, cached = np.zeros(1, np.int32), np.zeros(1, np.int32)
    rc = G.k3g_state_load(path.encode(), _ip(fp), _ip(seq), len(seq), _ip(nseq), dks.ptr, kper,
                          s["n_bound"], dlat.ptr, drope.ptr, s["n_mla"], cap, 512, 64,
                          _ip(cached))
    return rc, dict(ks=dks.numpy(), lat=dlat.numpy(), rope=drope.numpy(),
                    seq=seq[: nseq[0]], cached=int(cached[0]))


def test_round_trip_is_exact(ctx, state):
    G, path, s = state
    rc, got = _load(ctx, G, path, s)
    assert rc == 0 and got["cached"] == s["cached"]
    assert np.array_equal(got["seq"], s["seq"])
    assert np.array_equal(got["ks"], s["ks"])
    c = s["cached"]
    assert np.array_equal(got["lat"][:, :c], s["lat"][:, :c])
    assert np.array_equal(got["rope"][:, :c], s["rope"][:, :c])
    assert not got["lat"][:, c:].any()  # only the occupied positions travel


def test_header_is_the_reference_layout_with_version_4(state):
    _, path, s = state
    hd = np.fromfile(path, dtype=HDR, count=1)[0]
    assert HDR.itemsize == 104
    assert hd["magic"] == b"K3ST" and hd["version"] == 4
    assert np.array_equal(hd["fp"], FP)
    assert (hd["n_bound"], hd["n_mla"], hd["cached"], hd["nseq"]) == (3, 2, 37, 45)
    assert (hd["kper"], hd["kvpp"], hd["ropepp"]) == (1000, 512, 64)
    payload = 45 * 4 + 3 * 1000 * 4 + 2 * 37 * 512 * 2 + 2 * 37 * 64 * 2
    assert os.path.getsize(path) == 104 + payload


def test_resumed_cache_may_be_larger(ctx, state):
    G, path, s = state
    rc, got = _load(ctx, G, path, s, cap=80)
    c = s["cached"]
    assert rc == 0 and np.array_equal(got["lat"][:, :c], s["lat"][:, :c])


def test_refusals(ctx, state, tmp_path):
    G, path, s = state
    raw = open(path, "rb").read()
    assert _load(ctx, G, path, s, fp=FP + 1)[0] == -1          # another architecture
    assert _load(ctx, G, path, s, kper=999)[0] == -1           # another geometry
    assert _load(ctx, G, path, s, cap=20)[0] == -1             # cache too small
    bad = tmp_path / "bad.k3state"
    for data in (raw[:-1],                                     # truncated
                 raw + b"\0",                                  # longer than described
                 raw[:3000] + bytes([raw[3000] ^ 1]) + raw[3001:],  # one damaged byte
                 raw[:4] + (3).to_bytes(4, "little") + raw[8:]):    # version 3
        bad.write_bytes(data)
        assert _load(ctx, G, str(bad), s)[0] == -1
