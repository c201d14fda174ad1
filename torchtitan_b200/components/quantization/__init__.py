"""Float8 and MXFP8 training converters (parity: reference
``components/quantization/{float8,mx,utils}.py``).

A converter swaps matching ``Linear`` layers (FQN filter, both dims divisible
by 16 -- 32 for MX) for a quantized-training subclass.  Each GEMM of forward
and backward multiplies operands quantized along their contraction
dimension, as the recipes prescribe:

* forward ``y = x W^T``: x and W blocked along ``in``;
* dgrad ``dx = dy W``: dy and W blocked along ``out``;
* wgrad ``dW = dy^T x``: dy and x blocked along tokens.

The operands are quantized to the exact FP8/E8M0 codes and multiplied by the
bf16 tcgen05 GEMM on their dequantized values (numerically the block-scaled
product; the FP8 tensor-core kernel, ``kind::mxf8f6f4``, is not built yet).
"""
from .float8 import Float8LinearConverter
from .mx import MXFP8Converter
from .utils import module_filter

__all__ = ["Float8LinearConverter", "MXFP8Converter", "module_filter"]
