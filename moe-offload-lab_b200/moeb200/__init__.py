"""moeb200: the MoE-layer hot path of moelab (routing, dispatch, grouped expert products, combine)
as hand-written sm_100a CUDA behind a C ABI (include/moeb200.h), with thin torch-facing wrappers.

There is no CPU or torch fallback: every compute entry point runs libmoeb200's kernels and raises
MoeB200Error when the library is missing or a call is refused.
"""

from ._lib import MoeB200Error, lib
from .format import encode_record, record_layout, views
from .kernels import expert_ffn_int4, grouped_ffn_float, grouped_ffn_int4, grouped_ffn_int8
from .ops import PolicySpec
from .runtime import B200Experts, B200Router, B200Runtime, install

__all__ = ["MoeB200Error", "lib", "encode_record", "record_layout", "views", "expert_ffn_int4",
           "grouped_ffn_float", "grouped_ffn_int4", "grouped_ffn_int8", "PolicySpec", "B200Experts",
           "B200Router", "B200Runtime", "install"]
