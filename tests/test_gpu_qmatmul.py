"""GPU parity tests: the CUDA path (through the C ABI) against the CPU oracle.

Bars: bit-exact for integer work (INT8 quantisation, W8A8 products, weight
dequantisation); normwise max relative error <= 1e-3 (max|y - ref| /
max|ref|) for f32-activation block formats, whose reference route is
dequantise-to-f32 + f32 GEMV/GEMM.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from tests.helpers import max_rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-3  # max relative error for f32-accumulated outputs


def _sb():
    import synapse_b200 as sb
    return sb


@pytest.fixture(scope="module")
def rng():
    return np.random.default_rng(1234)


def cu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# ---------------------------------------------------------------------------
# a1: per-channel activation quantisation (bit-exact)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("rows,cols", [(1, 1), (1, 8), (3, 7), (16, 1024), (5, 3072),
                                       (2, 14336), (33, 100)])
def test_quantize_per_channel_bit_exact(rng, rows, cols):
    sb = _sb()
    x = rng.normal(0, 1, rows * cols).astype(np.float32)
    x[: cols] *= 100.0
    if rows > 2:
        x[cols:2 * cols] = 0.0  # an all-zero channel -> scale 1
    q, s = sb.quantize_per_channel_int8(cu(x), rows, cols)
    torch.cuda.synchronize()
    st, qo, so = oracle.quantize_per_channel_int8(x, rows, cols)
    assert st == 0
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))


def test_quantize_clamp_kat_on_gpu(kat):
    sb = _sb()
    k = kat["quantize_clamp"]
    q, s = sb.quantize_per_channel_int8(cu(np.array(k["input"], np.float32)), 1, 8)
    q = q.cpu().numpy()
    assert s.item() == k["scale"]
    for idx, val in k["pinned"].items():
        assert q[int(idx)] == val


def test_quantize_invalid_arg():
    sb = _sb()
    with pytest.raises(sb.SynapseError) as e:
        sb.quantize_per_channel_int8(cu(np.zeros(4, np.float32)), 0, 4)
    assert e.value.status == 2


@pytest.mark.parametrize("n,k", [(1, 1), (7, 13), (64, 128), (3072, 1024)])
def test_quantize_weights_bit_exact(rng, n, k):
    sb = _sb()
    w = rng.normal(0, 0.02, n * k).astype(np.float32)
    if n > 2:
        w[k:2 * k] = 0.0
    q, s = sb.quantize_weights_int8(cu(w), n, k)
    qo, so = oracle.quantize_weights_int8(w, n, k)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(s.cpu().numpy(), so)


# ---------------------------------------------------------------------------
# a2/a3: syn_qgemm_int8 on the reference's [K,N] layout (bit-exact)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (1, 1024, 1024), (1, 33, 1000), (2, 64, 64),
                                   (4, 256, 64), (7, 13, 5), (16, 3072, 1024), (17, 33, 25),
                                   (17, 96, 1536), (64, 64, 64), (128, 128, 512),
                                   (40, 200, 2100)])
def test_qgemm_int8_bit_exact(rng, m, n, k):
    sb = _sb()
    a = rng.integers(-127, 128, m * k).astype(np.int8)
    b = rng.integers(-128, 128, k * n).astype(np.int8)
    sa = np.abs(rng.normal(0, 0.01, m)).astype(np.float32)
    sbv = np.abs(rng.normal(0, 0.01, n)).astype(np.float32)
    c = sb.qgemm_int8(m, n, k, cu(a), cu(b), cu(sa), cu(sbv)).cpu().numpy()
    st, co = oracle.qgemm_int8(m, n, k, a, b, sa, sbv)
    assert st == 0
    assert np.array_equal(c.view(np.uint32), co.view(np.uint32)), \
        np.max(np.abs(c - co))


def test_qgemm_int8_strided(rng):
    # lda > k, ldb > n, ldc > n through the raw C entry point
    sb = _sb()
    m, n, k, lda, ldb, ldc = 3, 40, 70, 80, 48, 41
    a = rng.integers(-127, 128, m * lda).astype(np.int8)
    b = rng.integers(-127, 128, k * ldb).astype(np.int8)
    sa = np.abs(rng.normal(0, 0.01, m)).astype(np.float32)
    sbv = np.abs(rng.normal(0, 0.01, n)).astype(np.float32)
    da, db, dsa, dsb = cu(a), cu(b), cu(sa), cu(sbv)
    dc = torch.full((m * ldc,), 7.0, device="cuda")
    import ctypes
    st = sb.lib.syn_cuda_qgemm_int8(m, n, k, ctypes.c_void_p(da.data_ptr()), lda,
                                    ctypes.c_void_p(db.data_ptr()), ldb,
                                    ctypes.c_void_p(dc.data_ptr()), ldc,
                                    ctypes.c_void_p(dsa.data_ptr()),
                                    ctypes.c_void_p(dsb.data_ptr()), None)
    assert st == 0
    torch.cuda.synchronize()
    c = dc.cpu().numpy().reshape(m, ldc)
    a2 = a.reshape(m, lda)[:, :k]
    b2 = b.reshape(k, ldb)[:, :n]
    _, co = oracle.qgemm_int8(m, n, k, a2, b2, sa, sbv)
    assert np.array_equal(c[:, :n], co.reshape(m, n))
    assert np.all(c[:, n:] == 7.0)


# ---------------------------------------------------------------------------
# Weight handles: repack + bit-exact dequant hook
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("fmt", ["Q4_0", "Q8_0", "Q4_K", "Q6_K"])
def test_dequant_bit_exact_incl_subnormal_scales(ctx, rng, fmt):
    sb = _sb()
    from synapse_b200 import synth
    n, k = 33, 512
    f = sb.QFormat[fmt]
    blocks, _ = synth.gen_weight(f, n, k, rng)
    # force some subnormal f16 scales (converter.rs halves them)
    bsz = {"Q4_0": 18, "Q8_0": 34, "Q4_K": 144, "Q6_K": 210}[fmt]
    off = {"Q4_0": 0, "Q8_0": 0, "Q4_K": 0, "Q6_K": 208}[fmt]
    view = blocks.reshape(-1, bsz)
    for i in range(0, view.shape[0], 5):
        view[i, off:off + 2] = np.array([0x0001 + 37 * i % 0x3FF], np.uint16).view(np.uint8)
    w = sb.QuantizedWeight(ctx, f, blocks, n, k)
    got = w.dequant().reshape(-1)
    st, ref = oracle.dequant(fmt, blocks, n * k)
    assert st == 0
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_int8_dequant_bit_exact(ctx, rng):
    sb = _sb()
    n, k = 40, 70
    q = rng.integers(-128, 128, (k, n)).astype(np.int8)
    s = np.abs(rng.normal(0, 0.01, n)).astype(np.float32)
    w = sb.QuantizedWeight(ctx, sb.QFormat.INT8_KN, q, n, k, s)
    got = w.dequant()
    ref = (q.T.astype(np.float32) * s[:, None]).astype(np.float32)
    assert np.array_equal(got, ref)


def test_upload_shape_errors(ctx):
    sb = _sb()
    with pytest.raises(sb.SynapseError) as e:
        sb.QuantizedWeight(ctx, sb.QFormat.Q4_K, np.zeros(144 * 4, np.uint8), 4, 128)
    assert e.value.status == 4


# ---------------------------------------------------------------------------
# INT8 weight handle (QuantizedLinear::forward) -- bit-exact W8A8
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("m,n,k", [(1, 1024, 1024), (1, 3072, 1024), (1, 1024, 3072),
                                   (2, 100, 70), (3, 64, 64), (5, 33, 1000), (16, 2048, 1024),
                                   (17, 128, 1536), (24, 96, 520)])
def test_int8_handle_bit_exact(ctx, rng, m, n, k):
    sb = _sb()
    q = rng.integers(-127, 128, (k, n)).astype(np.int8)
    s = np.abs(rng.normal(0, 0.01, n)).astype(np.float32)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = sb.QuantizedWeight(ctx, sb.QFormat.INT8_KN, q, n, k, s)
    y = w.matmul(cu(x)).cpu().numpy().reshape(-1)
    _, xq, xs = oracle.quantize_per_channel_int8(x, m, k)
    _, yo = oracle.qgemm_int8(m, n, k, xq, q, xs, s)
    assert np.array_equal(y.view(np.uint32), yo.view(np.uint32)), np.max(np.abs(y - yo))
    # forward_pre_quantized == forward (int8_linear.rs:335-364)
    y2 = w.matmul_pre_quantized(cu(xq), cu(xs), m).cpu().numpy().reshape(-1)
    assert np.array_equal(y2, y)


def test_quantized_linear_reference_cases(ctx, kat):
    sb = _sb()
    from tests.helpers import frobenius_rel, xorshift_vec
    for m, k, n, sx, sw, frob, mabs in kat["int8_linear"]["cases"]:
        x = xorshift_vec(m * k, sx)
        w = xorshift_vec(n * k, sw)
        ql = sb.QuantizedLinear.from_f32(ctx, w, n, k)
        y = ql.forward(cu(x), m).cpu().numpy()
        wq, ws = oracle.quantize_weights_int8(w, n, k)
        assert np.array_equal(ql.weights_int8, wq) and np.array_equal(ql.scales, ws)
        _, xq, xs = oracle.quantize_per_channel_int8(x, m, k)
        _, yo = oracle.qgemm_int8(m, n, k, xq, wq, xs, ws)
        assert np.array_equal(y, yo)
        ref = (x.reshape(m, k) @ w.reshape(n, k).T).reshape(-1)
        if frob is not None:
            assert frobenius_rel(y, ref) < frob
        if mabs is not None:
            assert np.max(np.abs(y - ref)) <= mabs
    mb = kat["int8_linear"]["memory_bytes"]
    ql = sb.QuantizedLinear.from_f32(ctx, xorshift_vec(mb["n"] * mb["k"], 42), mb["n"], mb["k"])
    assert ql.memory_bytes() == mb["expected"]


# ---------------------------------------------------------------------------
# Block formats (f32 activations): within 1e-3 of dequant + f32 matmul
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("fmt", ["Q4_0", "Q8_0", "Q4_K", "Q6_K"])
@pytest.mark.parametrize("m,n,k", [(1, 1024, 1024), (1, 3072, 2048), (1, 7, 256), (2, 100, 512),
                                   (4, 64, 1024), (16, 256, 512), (17, 64, 256)])
def test_block_formats_within_tol(ctx, rng, fmt, m, n, k):
    sb = _sb()
    from synapse_b200 import synth
    f = sb.QFormat[fmt]
    blocks, _ = synth.gen_weight(f, n, k, rng)
    x = synth.gen_activations(m, k, rng)
    w = sb.QuantizedWeight(ctx, f, blocks, n, k)
    y = w.matmul(cu(x)).cpu().numpy().reshape(-1)
    st, yo = oracle.block_matmul(fmt, m, n, k, x, blocks)
    assert st == 0
    for i in range(m):
        assert max_rel_err(y[i * n:(i + 1) * n], yo[i * n:(i + 1) * n]) <= TOL


@pytest.mark.parametrize("n,k", [(4, 32), (5, 64), (1024, 1024), (3, 4096), (4097, 2048)])
def test_q4_0_gemv_raw(rng, n, k):
    sb = _sb()
    from synapse_b200 import synth
    blocks, _ = synth.gen_weight(sb.QFormat.Q4_0, n, k, rng)
    a = rng.normal(0, 1, k).astype(np.float32)
    c = sb.q4_0_gemv(n, k, cu(a), cu(blocks)).cpu().numpy()
    st, co = oracle.q4_0_gemv(n, k, a, blocks)
    assert st == 0
    assert max_rel_err(c, co) <= TOL


def test_q4_0_gemv_shape_error():
    sb = _sb()
    with pytest.raises(sb.SynapseError) as e:
        sb.q4_0_gemv(4, 48, cu(np.zeros(48, np.float32)), cu(np.zeros(4 * 36, np.uint8)))
    assert e.value.status == 4


# ---------------------------------------------------------------------------
# The full decode sweep (configs[1], M=1): every format x N x K
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("fmt", ["INT8_KN", "Q4_0", "Q8_0", "Q4_K", "Q6_K"])
def test_full_sweep_m1(ctx, fmt):
    sb = _sb()
    from synapse_b200 import synth
    rng = np.random.default_rng(99)
    f = sb.QFormat[fmt]
    for n in synth.SWEEP_N:
        for k in synth.SWEEP_K:
            data, scales = synth.gen_weight(f, n, k, rng)
            x = synth.gen_activations(1, k, rng)
            w = sb.QuantizedWeight(ctx, f, data, n, k, scales)
            y = w.matmul(cu(x)).cpu().numpy().reshape(-1)
            if f == sb.QFormat.INT8_KN:
                _, xq, xs = oracle.quantize_per_channel_int8(x, 1, k)
                _, yo = oracle.qgemm_int8(1, n, k, xq, data, xs, scales)
                assert np.array_equal(y, yo), (n, k)
            else:
                _, yo = oracle.block_matmul(fmt, 1, n, k, x, data)
                assert max_rel_err(y, yo) <= TOL, (n, k, max_rel_err(y, yo))
            w.close()
