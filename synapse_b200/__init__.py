"""synapse_b200 -- B200 (sm_100a) CUDA backend for Synapse's quantized-matmul
hot path, exposed through a C ABI (include/synapse_cuda.h) and mirrored here
in Python with the names of the reference's safe wrappers
(crates/synapse-core/src/lib.rs: quantize_per_channel_int8, qgemm_int8,
q4_0_gemv), of its INT8 layer (QuantizedLinear) and of its decoder-only LM
(Model: QuantizedCausalLM / CausalLM with the KV cache in HBM).
"""
from ._lib import load as _load

lib = _load()

from .api import (  # noqa: E402
    QFormat,
    SynapseError,
    Context,
    QuantizedWeight,
    QuantizedLinear,
    capability_summary,
    quantize_per_channel_int8,
    quantize_weights_int8,
    qgemm_int8,
    q4_0_gemv,
    row_bytes,
    rope_tables,
    rmsnorm,
    add_rmsnorm,
    swiglu,
    argmax,
    KVCache,
    attention_decode,
    attention_prefill,
    Model,
    tp_unique_id,
    tp_shard_linear,
)

__all__ = ["lib", "QFormat", "SynapseError", "Context", "QuantizedWeight", "QuantizedLinear",
           "capability_summary", "quantize_per_channel_int8", "quantize_weights_int8",
           "qgemm_int8", "q4_0_gemv", "row_bytes", "rope_tables", "rmsnorm", "add_rmsnorm",
           "swiglu", "argmax", "KVCache", "attention_decode", "attention_prefill", "Model", "tp_unique_id", "tp_shard_linear"]
