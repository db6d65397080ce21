"""CPU tests: the C-ABI library loads and exports every declared symbol."""
import ctypes
import glob
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(syn_cuda_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    import synapse_b200
    from synapse_b200 import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = declared_symbols()
    assert len(names) >= 14
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding declares every exported entry point
    assert names <= set(_lib.SIGNATURES), names - set(_lib.SIGNATURES)
    assert synapse_b200.lib is not None


def test_capability_and_status_strings():
    import synapse_b200 as sb
    cap = sb.capability_summary()
    assert cap["simd_backend"] == 3 and cap["abi_version"] == 1
    assert cap["feature_bits"] & (1 << 4) and cap["feature_bits"] & (1 << 5)
    assert sb.lib.syn_cuda_status_string(4) == b"shape mismatch"


def test_null_pointer_and_zero_size_checks_need_no_gpu():
    # exports.zig:1326-1331 order: null pointers first, then zero size -> OK.
    import synapse_b200 as sb
    L = sb.lib
    assert L.syn_cuda_qgemm_int8(1, 1, 1, None, 1, None, 1, None, 1, None, None, None) == 1
    one = ctypes.c_void_p(8)
    assert L.syn_cuda_qgemm_int8(0, 1, 1, one, 1, one, 1, one, 1, one, one, None) == 0
    assert L.syn_cuda_q4_0_gemv(4, 48, one, one, one, None) == 4
    assert L.syn_cuda_q4_0_gemv(0, 48, one, one, one, None) == 0
    assert L.syn_cuda_quantize_per_channel_int8(one, 0, 4, one, one, None) == 2
    assert L.syn_cuda_weight_upload(None, 0, None, 1, 1, None, None) == 1
    assert L.syn_cuda_qmatmul(None, None, None, 1, None, None) == 1
