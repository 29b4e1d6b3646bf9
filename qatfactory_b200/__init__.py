"""qatfactory_b200: QATFactory's fake-quantization path as sm_100a (B200) CUDA kernels.

``qatfactory_b200.quant`` is the drop-in for ``qatfactory.quant``; the kernels live in
``libqatf.so`` (C ABI declared in include/qatf.h) and are bound by ``_native``.
"""

__version__ = "0.1.0"
