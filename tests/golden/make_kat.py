"""Writes tests/golden/kat.json: the known-answer vectors and test shapes that
eren23/synapse's own test suites hold for the quantized-matmul path.

The reference (Zig + Rust) has no toolchain in this build environment, so the
vectors are transcribed from the reference test sources, each entry naming the
file:line it comes from (paths relative to the reference's `synapse/` root).
Run `python tests/golden/make_kat.py` to regenerate the file.
"""
import json
import os

KAT = {
    "quantize_clamp": {
        "source": "zig/tests/test_quantize.zig:225-246",
        "input": [100.0, -100.0, 50.0, -50.0, 0.0, 127.0, -127.0, 1.0],
        "scale": 1.0,
        # indices the reference test asserts, with their expected int8 values
        "pinned": {"0": 100, "1": -100, "5": 127, "6": -127},
        "range": [-127, 127],
    },
    "quantize_zero_channel": {
        "source": "zig/src/ops/quantize.zig:28-32 (all-zeros channel -> scale 1.0, q = 0)",
        "input": [0.0] * 16,
        "scale": 1.0,
    },
    "q8_0_block": {
        "source": "crates/synapse-inference/src/weight_loading/gguf.rs:701-722",
        "scale_bits": 0x3800,
        "quants": list(range(1, 33)),
        "expected": [0.5 * q for q in range(1, 33)],
        "tol": 1e-4,
    },
    "q4_0_block": {
        "source": "crates/synapse-inference/src/weight_loading/gguf.rs:790-821",
        "delta_bits": 0x3C00,
        "bytes": [0x10] * 16,
        # element 2i = low nibble - 8, element 2i+1 = high nibble - 8
        "expected": [-8.0, -7.0] * 16,
        "tol": 1e-3,
    },
    "qmatmul_shapes": {
        "source": "zig/tests/test_qmatmul.zig:126-159",
        # (m, n, k) as passed to checkQMatmul(allocator, m, n, k, tol)
        "shapes": [[8, 8, 8], [64, 64, 64], [128, 128, 512], [512, 512, 512],
                   [7, 13, 5], [17, 33, 25], [1, 1, 1], [4, 256, 64]],
        "lcg": {"mul": 1103515245, "add": 12345, "seed_a": 42, "seed_b": 137,
                "source": "zig/tests/test_qmatmul.zig:16-24"},
        "tiled_vs_naive_rel": 1e-5,
        "frobenius_vs_f32": 0.01,
    },
    "int8_linear": {
        "source": "crates/synapse-inference/src/quantization/primitives/int8_linear.rs:232-373",
        # (m, k, n, seed_x, seed_w, frobenius_tol, max_abs_tol or null)
        "cases": [[4, 16, 8, 42, 123, 0.1, None], [32, 128, 64, 777, 999, 0.1, None],
                  [1, 512, 512, 314, 159, 0.1, 0.5], [1, 256, 256, 2025, 2026, None, 0.5]],
        "single_element": {"w": 2.0, "x": 3.0, "expected": 6.0, "rel_tol": 0.1},
        "pre_quantized": {"m": 8, "k": 64, "n": 32, "seed_x": 555, "seed_w": 666, "tol": 1e-6},
        "memory_bytes": {"n": 64, "k": 128, "expected": 64 * 128 + 64 * 4},
    },
    "q4_0_gemv_shape_error": {
        "source": "zig/src/ffi/exports.zig:1614-1628 (k % 32 != 0 -> SYN_ERR_SHAPE_MISMATCH=4)",
        "k": 48, "status": 4,
    },
}

if __name__ == "__main__":
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kat.json")
    with open(out, "w") as f:
        json.dump(KAT, f, indent=1)
    print("wrote", out)
