"""synapse_b200 -- B200 (sm_100a) CUDA backend for Synapse's quantized-matmul
hot path, exposed through a C ABI (include/synapse_cuda.h) and mirrored here
in Python with the names of the reference's safe wrappers
(crates/synapse-core/src/lib.rs: quantize_per_channel_int8, qgemm_int8,
q4_0_gemv), of its INT8 layer (QuantizedLinear) and of its decoder-only LM
(Model: QuantizedCausalLM / CausalLM with the KV cache in HBM).

The public names load lazily: `synapse_b200.synth` and `synapse_b200.formats`
(input generators, format sizes) need neither torch nor the CUDA library,
while the first use of any other name (`lib`, `Context`, `QuantizedWeight`,
...) loads libsynapse_cuda.so and raises ImportError if it is missing -- there
is no CPU fallback.
"""
_API = ("QFormat", "SynapseError", "Context", "QuantizedWeight", "QuantizedLinear",
        "capability_summary", "quantize_per_channel_int8", "quantize_weights_int8",
        "qgemm_int8", "q4_0_gemv", "row_bytes", "rope_tables", "rmsnorm", "add_rmsnorm",
        "swiglu", "argmax", "KVCache", "attention_decode", "attention_prefill", "Model",
        "tp_unique_id", "tp_shard_linear", "GGUFFile", "SafetensorsFile", "gguf_runner_name",
        "quantize_weights_int8_half")

__all__ = ["lib"] + list(_API)


def __getattr__(name):
    if name == "lib":
        from ._lib import load
        lib = load()
        globals()["lib"] = lib
        return lib
    if name in _API:
        from . import api
        globals()["lib"] = __getattr__("lib") if "lib" not in globals() else globals()["lib"]
        val = getattr(api, name)
        globals()[name] = val
        return val
    raise AttributeError(f"module 'synapse_b200' has no attribute {name!r}")
