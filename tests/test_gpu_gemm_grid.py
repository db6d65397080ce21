"""The whole BASELINE config-2 grid at M > 1 through the product path
(QuantizedWeight.matmul -> syn_cuda_qmatmul): N in {1024, 3072, 4096, 11008,
14336} x K in {1024, 2048, 4096} x M in {16, 128, 512} x the five formats,
225 cases, each through whichever kernel the dispatcher picks (GEMV,
swapped-operand GEMM, 128-token tiles, k_qgemm_tm).

The C oracle needs minutes per large case on one core, so the checks use
the same arithmetic through numpy, pinned to the C oracle on one small case
per format in this file:
  INT8 (W8A8, bit-exact): activations quantised by the oracle
    (quantize.zig:12-47); the int32 dot products per 512-wide K chunk are
    exact in float64; then the reference's f32 epilogue in its order
    (qmatmul.zig:52-98): M <= 16 one accumulator, f32(acc) * sa * sb; M > 16
    C = 0 and C += f32(chunk) * sa * sb per chunk in K order.
  Block formats (normwise max relative error per output row <= 1e-3): the
    oracle's bit-exact dequantisation (gguf.rs:255-487) times x in float64.
    The reference's f32 sgemm differs from that by f32 summation error only
    (about 1e-6 here), three orders of magnitude under the bar.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from tests.helpers import max_rel_err

TOL = 1e-3
GRID_N = (1024, 3072, 4096, 11008, 14336)
GRID_K = (1024, 2048, 4096)
GRID_M = (16, 128, 512)


def int8_reference(xq, xs, q, sb, m, n, k):
    xq = xq.reshape(m, k).astype(np.float64)
    qf = q.reshape(k, n).astype(np.float64)
    sa = xs.astype(np.float32)[:, None]
    sbv = sb.astype(np.float32)[None, :]
    if m <= 16:
        acc = (xq @ qf).astype(np.float32)
        return (acc * sa).astype(np.float32) * sbv
    c = np.zeros((m, n), np.float32)
    for c0 in range(0, k, 512):
        acc = (xq[:, c0:c0 + 512] @ qf[c0:c0 + 512]).astype(np.float32)
        c = (c + ((acc * sa).astype(np.float32) * sbv).astype(np.float32)).astype(np.float32)
    return c


@pytest.mark.parametrize("m", [16, 40])
def test_int8_reference_model_matches_c_oracle(m):
    rng = np.random.default_rng(m)
    n, k = 96, 1536
    q = rng.integers(-127, 128, (k, n)).astype(np.int8)
    s = np.abs(rng.normal(0, 0.01, n)).astype(np.float32)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    _, xq, xs = oracle.quantize_per_channel_int8(x, m, k)
    _, yo = oracle.qgemm_int8(m, n, k, xq, q, xs, s)
    y = int8_reference(xq, xs, q, s, m, n, k)
    assert np.array_equal(y.reshape(-1).view(np.uint32), yo.view(np.uint32))


@pytest.mark.parametrize("fmt", ["Q4_0", "Q8_0", "Q4_K", "Q6_K"])
def test_block_reference_model_matches_c_oracle(fmt):
    import synapse_b200 as sb
    from synapse_b200 import synth
    rng = np.random.default_rng(3)
    m, n, k = 20, 64, 512
    blocks, _ = synth.gen_weight(sb.QFormat[fmt], n, k, rng)
    x = synth.gen_activations(m, k, rng)
    _, yo = oracle.block_matmul(fmt, m, n, k, x, blocks)
    w = oracle.dequant(fmt, blocks, n * k)[1].reshape(n, k).astype(np.float64)
    y = x.astype(np.float64) @ w.T
    assert np.max(np.abs(y - yo.reshape(m, n))) <= 1e-5 * np.max(np.abs(y))


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["INT8_KN", "Q4_0", "Q8_0", "Q4_K", "Q6_K"])
def test_config2_grid(ctx, fmt):
    import synapse_b200 as sb
    from synapse_b200 import synth
    f = sb.QFormat[fmt]
    worst = {}
    for n in GRID_N:
        for k in GRID_K:
            rng = np.random.default_rng(n * 31 + k)
            data, scales = synth.gen_weight(f, n, k, rng)
            w = sb.QuantizedWeight(ctx, f, data, n, k, scales)
            if f != sb.QFormat.INT8_KN:
                wd = oracle.dequant(fmt, data, n * k)[1].reshape(n, k).astype(np.float64)
            for m in GRID_M:
                x = synth.gen_activations(m, k, rng)
                y = w.matmul(torch.from_numpy(x).cuda()).cpu().numpy().reshape(m, n)
                if f == sb.QFormat.INT8_KN:
                    _, xq, xs = oracle.quantize_per_channel_int8(x, m, k)
                    ref = int8_reference(xq, xs, data, scales, m, n, k)
                    bad = int(np.sum(y.view(np.uint32) != ref.view(np.uint32)))
                    assert bad == 0, f"{m}x{n}x{k}: {bad} outputs differ"
                else:
                    ref = x.astype(np.float64) @ wd.T
                    err = max(max_rel_err(y[i], ref[i]) for i in range(m))
                    worst[(m, n, k)] = err
                    assert err <= TOL, f"{m}x{n}x{k}: {err}"
            w.close()
    if worst:
        key = max(worst, key=worst.get)
        print(f"{fmt}: worst normwise row error {worst[key]:.3e} at MxNxK {key}")
