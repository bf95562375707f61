"""actune_b200: B200-native (sm_100a) group-64 packed-integer linear for ActTune banks.

Public surface mirrors the reference package's hot path:

* ``actune_b200.kernels.grouped``: GroupedLinear, GroupedPaddedLinear, pack_rows,
  extension, reuse_mlp_temporary, shared_activation_scope
* ``actune_b200.kernels.quantizers``: weight_codes and the codebook helpers
* ``actune_b200.kernels.tuning``: bit-exact tile selection
* ``actune_b200.layers``: install_bank, ResidentLinear, BankRuntime, tensor_storage_bytes
* ``actune_b200.precision``: precision_profile, active_precision_profile, SharedBank
* ``actune_b200.graph``: GraphReplay
* ``actune_b200.ops``: tensor-level calls of the C ABI (include/actune_b200.h)

All arithmetic runs in libactune_b200.so (built by ``python -m actune_b200.build``).
"""
from .precision import CONFIGURATIONS, SharedBank, active_precision_profile, precision_profile  # noqa: F401

__version__ = "0.1.0"
