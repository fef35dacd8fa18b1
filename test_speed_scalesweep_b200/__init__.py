"""B200 (sm_100a) scale-sweep NVFP4 activation quantizer.

Drop-in for the reference's ``bench_kernel`` modules:

* :mod:`.scalesweep_mse_nvfp4_utils`            -- ``scalesweep_mse`` / ``scalesweep_mse128``
* :mod:`.scalesweep_mse_reference_nvfp4_utils`  -- ``scalesweep_mse_reference``
* :mod:`.custom`                                -- ``nvfp4_quant`` dispatcher
* :mod:`.global_scale`                          -- amax and the global-scale multiplier
* :mod:`.ops`                                   -- torch.library ops with fake impls
* :mod:`.sharded`                               -- row-sharded multi-GPU quantization

All compute runs in ``libscalesweep_b200.so`` (hand-written CUDA, C ABI in
``include/scalesweep_b200.h``).
"""
from .custom import create_fp4_output_tensors, nvfp4_quant  # noqa: F401

__version__ = "0.1.0"
