"""B200-native RepEncoder W8A8 hot path (sm_100a CUDA behind a C ABI).

Submodules mirror the reference modules they replace:

* ``w8a8_triton_kernels`` -- quantization/w8a8_triton_kernels.py
* ``w8a8_preprocess``     -- quantization/w8a8_preprocess.py
* ``quantization``        -- kernels/quantization.py
* ``rep_encoder_fusion``  -- kernels/rep_encoder_fusion.py
* ``rep_encoder``         -- models.RepEncoder (fuse_mode "b200")

The CUDA library is loaded on first use (``baidu_cti_grab_b200._lib``); every
device entry point raises if it cannot be loaded -- there is no CPU fallback.
"""

__all__ = ["synth"]
