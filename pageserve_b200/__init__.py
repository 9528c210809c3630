"""pageserve_b200: B200-native (sm_100a) kernels for pageserve's decode-step hot path.

The operator modules mirror the reference's names and signatures:
``pageserve_b200.paged_attention`` (engine/paged_attention.py),
``pageserve_b200.quantization`` (engine/quantization.py),
``pageserve_b200.model`` (engine/model.py) and
``pageserve_b200.tensor_parallel`` (engine/tensor_parallel.py). Every compute
call goes through the C-ABI library ``libpageserve_b200.so`` (declared in
include/pageserve_b200.h); there is no CPU fallback.
"""

__version__ = "0.1.0"
