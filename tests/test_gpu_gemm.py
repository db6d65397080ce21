"""GPU parity of the tensor-core GEMM path (M >= 8 activation rows).

INT8 (W8A8, kind::i8): bit-exact against the oracle for M <= 16 (one int32
accumulator over K) and M > 16 (the reference's per-512-K-chunk float
epilogue). Block formats (fp16 operands, fp32 accumulation): normwise max
relative error <= 1e-3 against dequantise + f32 matmul, per output row.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from tests.helpers import max_rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-3


# Below 40 rows, weights of fewer than 4096 rows (24 rows: 8192) run the GEMV;
# the n >= 8192 cases keep the tensor-core GEMM covered at small M.
@pytest.mark.parametrize("m,n,k", [(8, 64, 64), (16, 3072, 1024), (17, 128, 1536), (33, 200, 520),
                                   (8, 8192, 512), (17, 8192, 512), (33, 8224, 256),
                                   (128, 1024, 4096), (130, 96, 2048), (512, 512, 1024)])
def test_gemm_int8_bit_exact(ctx, m, n, k):
    import synapse_b200 as sb
    rng = np.random.default_rng(m * 7 + n + k)
    q = rng.integers(-127, 128, (k, n)).astype(np.int8)
    s = np.abs(rng.normal(0, 0.01, n)).astype(np.float32)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    x[min(1, m - 1)] = 0.0  # an all-zero activation row (scale 1)
    w = sb.QuantizedWeight(ctx, sb.QFormat.INT8_KN, q, n, k, s)
    y = w.matmul(torch.from_numpy(x).cuda()).cpu().numpy().reshape(-1)
    _, xq, xs = oracle.quantize_per_channel_int8(x, m, k)
    _, yo = oracle.qgemm_int8(m, n, k, xq, q, xs, s)
    assert np.array_equal(y.view(np.uint32), yo.view(np.uint32)), np.max(np.abs(y - yo))
    w.close()


@pytest.mark.parametrize("fmt", ["Q4_0", "Q8_0", "Q4_K", "Q6_K"])
@pytest.mark.parametrize("m,n,k", [(8, 256, 512), (9, 4096, 512), (16, 1024, 1024),
                                   (9, 8192, 512), (24, 8320, 256), (48, 8192, 512),
                                   (48, 384, 1024), (64, 160, 2048), (65, 256, 512),
                                   (128, 3072, 2048), (300, 100, 1024), (512, 1024, 4096),
                                   (129, 4096, 512), (200, 300, 2048), (144, 256, 1024),
                                   (32, 4096, 2048), (13, 4160, 1280)])
def test_gemm_block_formats_within_tol(ctx, fmt, m, n, k):
    import synapse_b200 as sb
    from synapse_b200 import synth
    rng = np.random.default_rng(m + n + k)
    f = sb.QFormat[fmt]
    blocks, _ = synth.gen_weight(f, n, k, rng)
    x = synth.gen_activations(m, k, rng)
    w = sb.QuantizedWeight(ctx, f, blocks, n, k)
    y = w.matmul(torch.from_numpy(x).cuda()).cpu().numpy().reshape(m, n)
    st, yo = oracle.block_matmul(fmt, m, n, k, x, blocks)
    assert st == 0
    yo = yo.reshape(m, n)
    errs = [max_rel_err(y[i], yo[i]) for i in range(m)]
    assert max(errs) <= TOL, max(errs)
    if fmt in ("Q4_K", "Q6_K") and m > 32:
        # split fp16 operands (weights and tokens as hi + lo): f32-grade
        assert max(errs) <= 5e-5, max(errs)
    w.close()


@pytest.mark.parametrize("fmt", ["Q4_0", "Q8_0"])
@pytest.mark.parametrize("m,n,k", [(20, 8192, 544), (64, 256, 544), (130, 200, 96)])
def test_gemm_odd_block_count(ctx, fmt, m, n, k):
    """K with an odd number of 32-element blocks: the last stage fills half
    of its 128-byte swizzle atom (swapped kernel, short and full 128-row
    tiles)."""
    import synapse_b200 as sb
    from synapse_b200 import synth
    rng = np.random.default_rng(m + 3 * n + k)
    f = sb.QFormat[fmt]
    blocks, _ = synth.gen_weight(f, n, k, rng)
    x = synth.gen_activations(m, k, rng)
    w = sb.QuantizedWeight(ctx, f, blocks, n, k)
    y = w.matmul(torch.from_numpy(x).cuda()).cpu().numpy().reshape(m, n)
    st, yo = oracle.block_matmul(fmt, m, n, k, x, blocks)
    assert st == 0
    yo = yo.reshape(m, n)
    assert max(max_rel_err(y[i], yo[i]) for i in range(m)) <= TOL
    w.close()


def test_gemm_error_word_clear(ctx):
    import ctypes
    import synapse_b200 as sb
    v = ctypes.c_int32(-1)
    assert sb.lib.syn_cuda_context_get_error(ctx.handle, ctypes.byref(v)) == 0
    assert v.value == 0


@pytest.mark.parametrize("fmt", ["Q4_0", "Q4_K", "Q6_K"])
@pytest.mark.parametrize("scale", [1e6, 1e-6])
def test_gemm_block_formats_activation_range(ctx, fmt, scale):
    """Rows far outside fp16 range (and tiny rows) keep the 1e-3 bound: the
    fp16 operand is scaled per row by an exact power of two."""
    import synapse_b200 as sb
    from synapse_b200 import synth
    m, n, k = 24, 256, 512
    rng = np.random.default_rng(int(scale * 7) % 1000 + 3)
    f = sb.QFormat[fmt]
    blocks, _ = synth.gen_weight(f, n, k, rng)
    x = synth.gen_activations(m, k, rng)
    x[::2] *= np.float32(scale)
    w = sb.QuantizedWeight(ctx, f, blocks, n, k)
    y = w.matmul(torch.from_numpy(x).cuda()).cpu().numpy().reshape(m, n)
    st, yo = oracle.block_matmul(fmt, m, n, k, x, blocks)
    yo = yo.reshape(m, n)
    assert np.all(np.isfinite(y))
    errs = [max_rel_err(y[i], yo[i]) for i in range(m)]
    assert max(errs) <= TOL, max(errs)
    w.close()


_CROSS = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
import synapse_b200 as sb
from synapse_b200 import synth
fmt, m, n, k = sys.argv[2], int(sys.argv[3]), int(sys.argv[4]), int(sys.argv[5])
rng = np.random.default_rng(11)
f = sb.QFormat[fmt]
blocks, _ = synth.gen_weight(f, n, k, rng)
x = synth.gen_activations(m, k, rng)
ctx = sb.Context(0)
w = sb.QuantizedWeight(ctx, f, blocks, n, k)
y = w.matmul(torch.from_numpy(x).cuda()).cpu().numpy()
np.save(sys.argv[6], y)
"""


@pytest.mark.parametrize("fmt,m", [("Q4_0", 128), ("Q4_0", 129), ("Q8_0", 129), ("Q4_K", 129),
                                   ("Q6_K", 64)])
def test_gemm_tm_crossover_both_paths(fmt, m, tmp_path):
    """The same inputs through k_qgemm_tm and through the 128-token-tile
    kernel (SYN_GEMM_TM_MIN_ROWS forced each way, in fresh processes):
    both within 1e-3 of the oracle, and within 2e-3 of each other."""
    import os
    import subprocess
    import sys
    from synapse_b200 import synth
    import synapse_b200 as sb
    n, k = 4096, 512
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    outs = []
    for tm_min in ("1", "0"):
        out = str(tmp_path / f"y{tm_min}.npy")
        env = dict(os.environ, SYN_GEMM_TM_MIN_ROWS=tm_min, SYN_GEMM_MIN_ROWS="1")
        subprocess.run([sys.executable, "-c", _CROSS, root, fmt, str(m), str(n), str(k), out],
                       env=env, check=True, timeout=600)
        outs.append(np.load(out).reshape(m, n))
    rng = np.random.default_rng(11)
    blocks, _ = synth.gen_weight(sb.QFormat[fmt], n, k, rng)
    x = synth.gen_activations(m, k, rng)
    st, yo = oracle.block_matmul(fmt, m, n, k, x, blocks)
    yo = yo.reshape(m, n)
    for y in outs:
        assert max(max_rel_err(y[i], yo[i]) for i in range(m)) <= TOL
    assert max(max_rel_err(outs[0][i], outs[1][i]) for i in range(m)) <= 2 * TOL

