"""The reference's own gates, run through the B200 drop-ins.

tests/refgate/Makefile builds the reference's unmodified tests/unit/test_ops.c,
tests/unit/k3_model.c and benchmarks/bench_kernels.c against its unmodified
src/core/k3_ops.c, with k3_gpu_interpose.c linked ahead of it, so that every k3_kda_step,
k3_kda_layer and k3_mla_cached call -- the tests' own and those inside k3_decoder_layer_inc
and k3_mla -- runs on the GPU through include/k3_gpu.h (built here from the reference
checkout; the binaries and the fixtures they read travel in tests/refgate/_build).

  * test_ops: the per-op fixtures at the reference's MANIFEST tolerance (1e-5 absolute +
    1e-4 relative, elementwise), the recurrence, MLA and KDA layer fixtures and the two
    decoder-layer fixtures among them.
  * k3_model: the 13-layer tiny model's gates. Gates 1, 2 and 3 demand exact tokens
    (teacher forcing, greedy decode, incremental decode over the carried KDA state and MLA
    cache); 1b and 3b demand bit-identical logits and state between two schedules of the
    same tokens. With K3G_TOKENWISE=1 every multi-token call is run as one-token calls, and
    the whole verdict must read "ENGINE MATCHES THE REFERENCE EXACTLY". In the default
    (chunked) mode gate 3b compares a chunked prefill with token-by-token decoding, which
    agree within the tolerance but not to the bit; the tokens must still match exactly.
  * bench_kernels: the reference's microbenchmark in GPU mode (its MLA decode section runs
    through k3g_mla_cached); it must complete and its output must be the same bits at one
    and at all host threads.
"""
import os
import re
import subprocess

import pytest

pytestmark = pytest.mark.gpu

B = os.path.join(os.path.dirname(os.path.abspath(__file__)), "refgate", "_build")
FIX = os.path.join(B, "fixtures")
built = pytest.mark.skipif(not os.path.exists(os.path.join(B, "test_ops_gpu")),
                           reason="tests/refgate not built (needs the reference checkout)")


def _run(prog, *args, env=None, timeout=600):
    e = dict(os.environ)
    e.pop("K3G_TOKENWISE", None)
    e.update(env or {})
    r = subprocess.run([os.path.join(B, prog), *args], capture_output=True, text=True,
                       timeout=timeout, env=e, cwd=B)
    return r.returncode, r.stdout, r.stderr


def _routed(stderr):
    m = re.search(r"k3_kda_step (\d+), k3_kda_layer (\d+), k3_mla_cached (\d+)", stderr)
    assert m, stderr[-2000:]
    return tuple(int(x) for x in m.groups())


@built
def test_reference_op_tests_through_the_gpu():
    rc, out, err = _run("test_ops_gpu", os.path.join(FIX, "ops"))
    print(out)
    step, kda, mla = _routed(err)
    assert step > 0 and kda > 0 and mla > 0, (step, kda, mla)
    m = re.search(r"(\d+) passed, (\d+) failed, (\d+) skipped", out)
    assert m, out[-2000:]
    passed, failed, skipped = (int(x) for x in m.groups())
    assert (failed, skipped) == (0, 0) and passed == 22 and rc == 0, out[-3000:]


@built
def test_reference_model_gates_tokenwise_exact():
    rc, out, err = _run("k3_model_gpu", FIX, env={"K3G_TOKENWISE": "1"})
    print(out)
    _, kda, mla = _routed(err)
    assert kda > 0 and mla > 0
    assert "VERDICT: ENGINE MATCHES THE REFERENCE EXACTLY" in out and rc == 0, out[-3000:]


@built
def test_reference_model_gates_chunked_tokens_exact():
    rc, out, err = _run("k3_model_gpu", FIX)
    print(out)
    _, kda, mla = _routed(err)
    assert kda > 0 and mla > 0
    g1 = re.search(r"generated span\s*:\s*(\d+)/(\d+)", out)
    g2 = re.search(r"GATE 2\s+greedy decode\s*:\s*(\d+)/(\d+)", out)
    g3 = re.search(r"GATE 3\s+incremental\s*:\s*(\d+)/(\d+)", out)
    for g in (g1, g2, g3):
        assert g and g.group(1) == g.group(2), out[-3000:]
    assert "GATE 1b state reuse      : PASS" in out, out[-3000:]


@built
def test_reference_bench_kernels_gpu_mode():
    rc, out, err = _run("bench_kernels_gpu", timeout=1200)
    print(out)
    _, _, mla = _routed(err)
    assert mla > 0
    assert rc == 0 and "bit-identical" in out, out[-3000:]
