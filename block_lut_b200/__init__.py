"""block_lut_b200: the LUT-dequantised MoE expert forward of block_lut on B200 (sm_100a).

Python / PyTorch host code over ``libblut.so`` (C ABI in ``include/blut.h``):

* ``formats``        -- LUT formats, GPU encoders, bit-exact dequant, tiled layout
* ``moe``            -- ``LUTMoELayer``: one MoE layer per ``blut_moe_forward`` call
* ``quant_method``   -- vLLM plugin ``"lut"`` (reference ``vllm_lut/quant_method.py``)
* ``fast_moe``       -- ``fused_lut_moe`` (reference ``vllm_lut/fast_moe.py``)
* ``cuda_lut_gemv``  -- ``lut_gemv`` (reference ``vllm_lut/cuda_lut_gemv.py``)
* ``fused_kernel``   -- ``fused_lut_gemv`` (reference ``vllm_lut/fused_kernel.py``)
* ``quantizer``      -- ``LUTQuantizer``, ``decompress_blocklut`` (reference ``vllm_lut/quantizer.py``)
* ``moe_layer``      -- ``DeepseekV2MoE_LUT``, ``_routing`` (reference ``vllm_lut/moe_layer.py``)
* ``linear``         -- ``LUTLinear``: one weight matrix, any format and token count
* ``ep``             -- ``EPMoELayer``: expert parallelism over NCCL
* ``bitplanes``      -- progressive bit-plane tiers of Format R (``runtime/model_offload.py``)
* ``convert_checkpoint`` -- bf16 checkpoint -> LUT checkpoint (reference ``vllm_lut/convert_checkpoint.py``)
"""
from . import _lib
from .formats import LUTFormat, QuantizedMatrix, dequant, encode, encode_r, pack_tiled, tiled_bytes
from .moe import LUTExperts, LUTMoELayer, SharedExpert, router

__all__ = ["_lib", "LUTFormat", "QuantizedMatrix", "dequant", "encode", "encode_r", "pack_tiled", "tiled_bytes",
           "LUTExperts", "LUTMoELayer", "SharedExpert", "router"]
