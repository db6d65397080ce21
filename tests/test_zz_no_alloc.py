"""GPU test of syn_cuda_qmatmul_noalloc, the allocation-free GEMV entry point.

Some callers cannot allocate device memory while they run: a latency-critical
decode loop where an allocation could stall, a process whose device memory
belongs to an external pool or budget, or a plug-in host that forbids the
CUDA allocator. For them the library keeps the GEMV's scratch (split-K
partial sums and arrival counters) in one fixed device array. This test calls
that entry point through the C ABI and checks that it returns what
syn_cuda_qmatmul returns -- bit-exact for INT8, within 1e-3 relative error
for the block formats, the tolerances of the other GPU tests -- on two calls
in a row (the shared array keeps the previous call's contents), and that a
call needing more scratch than the array holds is refused.

The file name makes pytest collect it last.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _noalloc(sb, w, x, m, y):
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return sb.lib.syn_cuda_qmatmul_noalloc(w.handle, _ptr(x), m, _ptr(y), st)


def _rel(a, b):
    den = np.max(np.abs(b))
    return float(np.max(np.abs(a - b)) / den) if den > 0 else float(np.max(np.abs(a)))


@pytest.mark.parametrize("fmt,m,n,k", [
    ("Q4_0", 1, 1024, 4096),     # K split across CTAs: partials + counters used
    ("INT8_KN", 1, 1024, 4096),  # split, per-512 chunk integer partials
    ("Q6_K", 2, 3072, 2048),
    ("Q4_K", 1, 4096, 4096),
    ("INT8_KN", 20, 256, 1536),  # M > 16: the reference's chunked epilogue
    ("Q8_0", 1, 14336, 1024),    # no split
])
def test_noalloc_matches_qmatmul_twice(fmt, m, n, k):
    import synapse_b200 as sb
    from synapse_b200 import synth
    ctx = sb.Context(0)
    rng = np.random.default_rng(4321 + n + k + m)
    f = sb.QFormat[fmt]
    data, scales = synth.gen_weight(f, n, k, rng)
    w = sb.QuantizedWeight(ctx, f, data, n, k, scales)
    for call in range(2):
        x = torch.from_numpy(synth.gen_activations(m, k, rng)).cuda()
        ref = w.matmul(x).cpu().numpy()
        y = torch.full((m, n), float("nan"), device="cuda")
        st = _noalloc(sb, w, x, m, y)
        assert st == 0, (call, st, sb.lib.syn_cuda_last_error())
        got = y.cpu().numpy()
        if f == sb.QFormat.INT8_KN:
            assert np.array_equal(got, ref), call
        else:
            assert _rel(got, ref) <= TOL, (call, _rel(got, ref))
    w.close()
    ctx.close()


def test_noalloc_rejects_oversized_scratch():
    import synapse_b200 as sb
    from synapse_b200 import synth
    ctx = sb.Context(0)
    rng = np.random.default_rng(7)
    n, k, m = 32768, 1024, 2048  # counters alone: 2048 x 1024 row groups x 4 B = 8 MiB
    data, _ = synth.gen_weight(sb.QFormat.Q4_0, n, k, rng)
    w = sb.QuantizedWeight(ctx, sb.QFormat.Q4_0, data, n, k)
    x = torch.zeros(m, k, device="cuda")
    y = torch.full((m, n), 7.0, device="cuda")
    assert _noalloc(sb, w, x, m, y) == 3  # SYN_ERR_OUT_OF_MEMORY
    torch.cuda.synchronize()
    assert bool(torch.all(y == 7.0))
    w.close()
    ctx.close()


@pytest.mark.parametrize("fmt", ["Q6_K", "Q8_0"])
def test_noalloc_near_the_limit(fmt):
    """Rows 1..16 of a 14336 x 4096 weight: the split-K partials grow with
    the rows until the fixed array no longer holds them. Accepted calls
    match syn_cuda_qmatmul; refused ones touch nothing."""
    import synapse_b200 as sb
    from synapse_b200 import synth
    ctx = sb.Context(0)
    rng = np.random.default_rng(99)
    n, k = 14336, 4096
    f = sb.QFormat[fmt]
    data, _ = synth.gen_weight(f, n, k, rng)
    w = sb.QuantizedWeight(ctx, f, data, n, k)
    accepted = []
    for m in range(1, 17):
        x = torch.from_numpy(synth.gen_activations(m, k, rng)).cuda()
        y = torch.full((m, n), 7.0, device="cuda")
        st = _noalloc(sb, w, x, m, y)
        if st == 3:
            torch.cuda.synchronize()
            assert bool(torch.all(y == 7.0)), m
            continue
        assert st == 0, (m, st, sb.lib.syn_cuda_last_error())
        ref = w.matmul(x).cpu().numpy()
        assert _rel(y.cpu().numpy(), ref) <= TOL, m
        accepted.append(m)
    assert accepted and accepted[0] == 1, accepted
    w.close()
    ctx.close()
