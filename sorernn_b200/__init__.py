"""B200-native (sm_100a) Gated DeltaNet token mixer: a drop-in for soreRNN's GDN op.

Public API (torch tensors on a CUDA device):
  * :func:`chunk_gated_delta_rule` — the op soreRNN calls at sore/model/gdn.py:166 (fwd + autograd bwd);
  * :func:`fused_recurrent_gated_delta_rule_step` — the single-token decode step on a resident state;
  * :mod:`sorernn_b200.seqsplit` — sequence-split long prefill across ranks.
The kernels live in the C-ABI library ``_lib/libgdn_b200.so`` (include/gdn_b200.h).
"""
from .gated_delta_rule import chunk_gated_delta_rule, fused_recurrent_gated_delta_rule_step  # noqa: F401
