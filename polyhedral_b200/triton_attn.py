"""Drop-in module name for the reference's ``gpu/triton_attn.py``: same public
function and kind constants.  No Triton is involved -- ``block_sparse_attention``
is the sm_100a tcgen05 kernel of csrc/attn.cu."""
from .attention import (CAUSAL, DILATED, FAR_STRIDED, LOCAL_STRIDED, SINKS,  # noqa: F401
                        TWOBAND, WINDOW, AttnPlan, block_sparse_attention, make_plan)
