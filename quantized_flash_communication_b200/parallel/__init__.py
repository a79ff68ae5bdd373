"""Cross-GPU communication: peer-mapped workspaces and the fused quantized all-reduce."""
from .symm_mem import SymmetricWorkspace, EmulatedWorkspaces, CommTimeoutError  # noqa: F401
from .quant_allreduce import QuantAllReduce, EmulatedQuantAllReduce  # noqa: F401
from .staged import staged_all_reduce  # noqa: F401
