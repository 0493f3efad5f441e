"""af2cuda: host-side mirror of alphafold2-webgpu's pair-stack operator API over
libaf2cuda.so (sm_100a CUDA kernels behind a C ABI).

The class and option names follow the reference's TypeScript exports
(src/index.ts) so parity tests read like the reference's own tests.
"""
from ._lib import Af2Error, RangeError, lib
from .attention import (AttentionGpu, AttentionInput, AttentionResult, AttentionWeights, NormalizedInputPairBias,
                        SeparatePairBias, attention_weight_count, attention_workspace_bytes,
                        encode_attention_tensors, encode_triangle_attention_tensors, pack_attention_weights)
from .block import encode_evoformer_pair_block_tensors
from .bundle import TriangleReferenceBundle, load_triangle_reference_bundle_from_files
from .device import Device
from .triangle import (TriangleGpuOptions, TriangleGpuResult, TriangleMultiplicationIncomingGpu,
                       TriangleMultiplicationOutgoingGpu, encode_triangle_multiplication,
                       encode_triangle_multiplication_tensors, triangle_weight_count, triangle_workspace_bytes)
from .opm import (OuterProductMeanGpu, OuterProductMeanInput, OuterProductMeanResult, OuterProductMeanWeights,
                  encode_outer_product_mean_tensors, linear_tensors, opm_weight_count, opm_workspace_bytes,
                  pack_outer_product_mean_weights, validate_outer_product_mean_input)
from .sharded import (PeerLost, PeerMonitor, comm_abort, comm_destroy, comm_init, comm_set_timeout, comm_unique_id,
                      encode_outer_product_mean_sharded_tensors, encode_triangle_multiplication_sharded_tensors,
                      rows_of)
from .transition import (Q8Matrix, TransitionGpu, TransitionInput, TransitionResult, TransitionWeights,
                         dequant_q8_tensors, encode_transition_tensors, pack_transition_weights,
                         transition_weight_count, transition_workspace_bytes, validate_transition_input)
from .tensor_store import (FileTensorStore, block_range, quantize_q8_block, read_tensor_range, tensor_byte_length,
                           tensor_elements, write_tensor_manifest)
from .weights import (encode_outer_product_mean_weight_tensors, encode_triangle_multiplication_weight_tensors,
                      opm_tensor_sizes, stored_weights, triangle_tensor_sizes)
from .types import (ORDER, TriangleMultiplicationInput, TriangleMultiplicationWeights, TriangleShape,
                    error_metrics, expected_weight_element_count, pack_weights, validate_triangle_input)

__all__ = [
    "Af2Error", "RangeError", "lib", "Device", "TriangleReferenceBundle", "load_triangle_reference_bundle_from_files",
    "TriangleGpuOptions", "TriangleGpuResult", "TriangleMultiplicationIncomingGpu", "TriangleMultiplicationOutgoingGpu",
    "encode_triangle_multiplication", "encode_triangle_multiplication_tensors", "triangle_weight_count",
    "triangle_workspace_bytes", "ORDER", "TriangleMultiplicationInput", "TriangleMultiplicationWeights",
    "TriangleShape", "error_metrics", "expected_weight_element_count", "pack_weights", "validate_triangle_input",
    "Q8Matrix", "TransitionGpu", "TransitionInput", "TransitionResult", "TransitionWeights", "dequant_q8_tensors",
    "encode_transition_tensors", "pack_transition_weights", "transition_weight_count", "transition_workspace_bytes",
    "validate_transition_input", "OuterProductMeanGpu", "OuterProductMeanInput", "OuterProductMeanResult",
    "OuterProductMeanWeights", "encode_outer_product_mean_tensors", "linear_tensors", "opm_weight_count",
    "opm_workspace_bytes", "pack_outer_product_mean_weights", "validate_outer_product_mean_input",
    "comm_destroy", "comm_init", "comm_unique_id", "encode_triangle_multiplication_sharded_tensors", "rows_of",
    "encode_outer_product_mean_sharded_tensors", "AttentionGpu", "AttentionInput", "AttentionResult",
    "AttentionWeights", "NormalizedInputPairBias", "SeparatePairBias", "attention_weight_count",
    "attention_workspace_bytes", "encode_attention_tensors", "encode_triangle_attention_tensors",
    "pack_attention_weights", "encode_evoformer_pair_block_tensors", "FileTensorStore", "block_range",
    "quantize_q8_block", "read_tensor_range", "tensor_byte_length", "tensor_elements", "write_tensor_manifest",
    "encode_outer_product_mean_weight_tensors", "encode_triangle_multiplication_weight_tensors", "opm_tensor_sizes",
    "stored_weights", "triangle_tensor_sizes", "PeerLost", "PeerMonitor", "comm_set_timeout", "comm_abort",
]
