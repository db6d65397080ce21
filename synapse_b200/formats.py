"""Weight formats of the quantized-matmul path and their storage sizes.

Plain Python with no native dependency, so that input generators and the CPU
legs of the benchmark can describe weights without loading the CUDA library.
Block layouts: GGUF Q4_0 / Q8_0 (32 elements, 18 / 34 bytes) and Q4_K / Q6_K
(256 elements, 144 / 210 bytes), as weight_loading/gguf.rs:255-487 reads
them; INT8_KN is the reference's transposed [K, N] int8 operand with f32
per-row scales (int8_linear.rs:7-18).
"""
import enum


class QFormat(enum.IntEnum):
    INT8_KN = 0
    Q4_0 = 1
    Q8_0 = 2
    Q4_K = 3
    Q6_K = 4


BLOCK = {QFormat.Q4_0: (32, 18), QFormat.Q8_0: (32, 34), QFormat.Q4_K: (256, 144),
         QFormat.Q6_K: (256, 210)}


def row_bytes(fmt, k):
    """Bytes of one K-element row in the reference's storage format; raises
    ValueError when K is not a whole number of blocks."""
    fmt = QFormat(fmt)
    if fmt == QFormat.INT8_KN:
        return k
    elems, nbytes = BLOCK[fmt]
    if k % elems:
        raise ValueError(f"K={k} is not a multiple of the {fmt.name} block ({elems})")
    return k // elems * nbytes
