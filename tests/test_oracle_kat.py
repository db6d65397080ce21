"""CPU tests: the oracle against the reference's own known-answer tests and
properties (tests/golden/kat.json), plus f16 conversion checks."""
import numpy as np
import pytest

from oracle import oracle
from tests.helpers import frobenius_rel, lcg_fill, max_rel_err, quantize_per_column_int8, \
    xorshift_vec


def test_f16_zig_is_ieee_and_rust_halves_subnormals():
    bits = np.arange(0, 1 << 16, dtype=np.uint16)
    ieee = bits.view(np.float16).astype(np.float32)
    zig = np.array([oracle.f16_zig(b) for b in bits], dtype=np.float32)
    rust = np.array([oracle.f16_rust(b) for b in bits], dtype=np.float32)
    fin = np.isfinite(ieee)
    assert np.array_equal(zig[fin].view(np.uint32), ieee[fin].view(np.uint32))
    assert np.all(np.isnan(zig[~fin & np.isnan(ieee)]))
    sub = ((bits >> 10) & 0x1F) == 0
    sub &= (bits & 0x3FF) != 0
    # converter.rs:21-30 starts its counter at 1: every subnormal is halved
    assert np.array_equal(rust[sub], (ieee[sub] * np.float32(0.5)).astype(np.float32))
    assert np.array_equal(rust[fin & ~sub].view(np.uint32), ieee[fin & ~sub].view(np.uint32))


def test_quantize_clamp_kat(kat):
    k = kat["quantize_clamp"]
    st, q, s = oracle.quantize_per_channel_int8(np.array(k["input"], np.float32), 1, 8)
    assert st == 0
    assert abs(s[0] - k["scale"]) <= 1e-7
    for idx, val in k["pinned"].items():
        assert q[int(idx)] == val
    assert q.min() >= k["range"][0] and q.max() <= k["range"][1]


def test_quantize_zero_channel(kat):
    k = kat["quantize_zero_channel"]
    st, q, s = oracle.quantize_per_channel_int8(np.array(k["input"], np.float32), 1, 16)
    assert st == 0 and s[0] == 1.0 and not q.any()


def test_quantize_invalid_args():
    st, _, _ = oracle.quantize_per_channel_int8(np.zeros(1, np.float32), 0, 1)
    assert st == 2


@pytest.mark.parametrize("channels,size", [(4, 16), (16, 64), (3, 1000)])
def test_quantize_roundtrip_and_symmetry(channels, size):
    # test_quantize.zig:57-222: per-channel round trip <= 0.5%, q(-x) = -q(x)
    x = lcg_fill(channels * size, 42, 10.0)
    st, q, s = oracle.quantize_per_channel_int8(x, channels, size)
    rec = (q.reshape(channels, size).astype(np.float32) * s[:, None]).reshape(-1)
    for c in range(channels):
        sl = slice(c * size, (c + 1) * size)
        assert np.max(np.abs(x[sl] - rec[sl])) / np.max(np.abs(x[sl])) <= 0.005
    _, qn, sn = oracle.quantize_per_channel_int8(-x, channels, size)
    assert np.array_equal(qn, -q) and np.array_equal(sn, s)


def test_q8_0_block_kat(kat):
    k = kat["q8_0_block"]
    blk = np.zeros(34, np.uint8)
    blk[0:2] = np.array([k["scale_bits"]], np.uint16).view(np.uint8)
    blk[2:] = np.array(k["quants"], np.int8).view(np.uint8)
    st, out = oracle.dequant("Q8_0", blk, 32)
    assert st == 0
    assert np.max(np.abs(out - np.array(k["expected"], np.float32))) < k["tol"]


def test_q4_0_block_kat(kat):
    k = kat["q4_0_block"]
    blk = np.zeros(18, np.uint8)
    blk[0:2] = np.array([k["delta_bits"]], np.uint16).view(np.uint8)
    blk[2:] = np.array(k["bytes"], np.uint8)
    st, out = oracle.dequant("Q4_0", blk, 32)
    assert st == 0
    assert np.max(np.abs(out - np.array(k["expected"], np.float32))) < k["tol"]


def test_q4_0_gemv_shape_error(kat):
    k = kat["q4_0_gemv_shape_error"]
    st, _ = oracle.q4_0_gemv(4, k["k"], np.zeros(k["k"], np.float32),
                             np.zeros(4 * 18 * 2, np.uint8))
    assert st == k["status"]


@pytest.mark.parametrize("shape", [[8, 8, 8], [64, 64, 64], [128, 128, 512], [7, 13, 5],
                                   [17, 33, 25], [1, 1, 1], [4, 256, 64], [512, 512, 512]])
def test_qmatmul_reference_suite(kat, shape):
    # zig/tests/test_qmatmul.zig:32-159: tiled vs naive <= 1e-5 relative and
    # INT8 vs f32 Frobenius <= 1%.
    m, n, k = shape
    cfg = kat["qmatmul_shapes"]
    a = lcg_fill(m * k, cfg["lcg"]["seed_a"])
    b = lcg_fill(k * n, cfg["lcg"]["seed_b"])
    ref = (a.reshape(m, k).astype(np.float64) @ b.reshape(k, n).astype(np.float64)).reshape(-1)
    _, aq, sa = oracle.quantize_per_channel_int8(a, m, k)
    bq, sb = quantize_per_column_int8(b, k, n)
    st, tiled = oracle.qgemm_int8(m, n, k, aq, bq, sa, sb)
    naive = oracle.naive_int8_gemm(m, n, k, aq, bq, sa, sb)
    assert st == 0
    rel = np.abs(tiled - naive) / np.maximum(np.abs(naive), 1e-6)
    assert rel.max() <= cfg["tiled_vs_naive_rel"]
    assert frobenius_rel(tiled, ref) <= cfg["frobenius_vs_f32"]


def test_qgemm_chunking_is_visible_above_16_rows():
    # M>16 sums float(acc_chunk) per 512-wide K chunk; M<=16 uses one int32
    # accumulator. With K=1536 the two differ in the last bits somewhere.
    rng = np.random.default_rng(7)
    m, n, k = 17, 64, 1536
    a = rng.integers(-127, 128, m * k).astype(np.int8)
    b = rng.integers(-127, 128, k * n).astype(np.int8)
    sa = np.abs(rng.normal(0, 0.01, m)).astype(np.float32)
    sb = np.abs(rng.normal(0, 0.01, n)).astype(np.float32)
    _, c = oracle.qgemm_int8(m, n, k, a, b, sa, sb)
    naive = oracle.naive_int8_gemm(m, n, k, a, b, sa, sb)
    assert not np.array_equal(c, naive)
    assert max_rel_err(c, naive) < 1e-6


@pytest.mark.parametrize("case", [0, 1, 2, 3])
def test_int8_linear_reference_cases(kat, case):
    # int8_linear.rs:232-312: QuantizedLinear::from_f32 then forward vs f32.
    m, k, n, sx, sw, frob, mabs = kat["int8_linear"]["cases"][case]
    x = xorshift_vec(m * k, sx)
    w = xorshift_vec(n * k, sw)
    wq, ws = oracle.quantize_weights_int8(w, n, k)
    _, xq, xs = oracle.quantize_per_channel_int8(x, m, k)
    _, y = oracle.qgemm_int8(m, n, k, xq, wq, xs, ws)
    ref = (x.reshape(m, k).astype(np.float32) @ w.reshape(n, k).T.astype(np.float32)).reshape(-1)
    if frob is not None:
        assert frobenius_rel(y, ref) < frob
    if mabs is not None:
        assert np.max(np.abs(y - ref)) <= mabs


def test_int8_linear_single_element(kat):
    c = kat["int8_linear"]["single_element"]
    wq, ws = oracle.quantize_weights_int8(np.array([c["w"]], np.float32), 1, 1)
    _, xq, xs = oracle.quantize_per_channel_int8(np.array([c["x"]], np.float32), 1, 1)
    _, y = oracle.qgemm_int8(1, 1, 1, xq, wq, xs, ws)
    assert abs(y[0] - c["expected"]) / c["expected"] < c["rel_tol"]


@pytest.mark.parametrize("fmt", ["Q4_0", "Q8_0", "Q4_K", "Q6_K"])
def test_block_matmul_close_to_float64(fmt):
    from synapse_b200 import synth
    from synapse_b200.api import QFormat
    rng = np.random.default_rng(3)
    n, k = 64, 512
    blocks, _ = synth.gen_weight(QFormat[fmt], n, k, rng)
    x = synth.gen_activations(3, k, rng)
    st, w = oracle.dequant(fmt, blocks, n * k)
    assert st == 0 and np.all(np.isfinite(w))
    st, y = oracle.sgemm_nt(3, n, k, x, w)
    ref = (x.astype(np.float64) @ w.reshape(n, k).T.astype(np.float64)).reshape(-1)
    assert max_rel_err(y, ref) < 1e-5


def test_q4_0_gemv_matches_dequant_route():
    # syn_q4_0_gemv (Zig f16) and the loader route (Rust f16) agree within
    # 1e-3 when no scale is subnormal; both are within f32 rounding of f64.
    from synapse_b200 import synth
    from synapse_b200.api import QFormat
    rng = np.random.default_rng(11)
    n, k = 37, 256
    blocks, _ = synth.gen_weight(QFormat.Q4_0, n, k, rng)
    x = rng.normal(0, 1, k).astype(np.float32)
    st, c = oracle.q4_0_gemv(n, k, x, blocks)
    assert st == 0
    st, y = oracle.block_matmul("Q4_0", 1, n, k, x, blocks)
    d = blocks.reshape(-1, 18)[:, 0:2].copy().view(np.uint16).reshape(-1)
    if not np.any(((d >> 10) & 0x1F) == 0):
        assert max_rel_err(c, y) < 1e-5
