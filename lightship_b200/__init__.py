"""lightship_b200 -- a B200 (sm_100a) CUDA backend for the LightShip inference engine.

The product is the C-ABI library ``liblightship_cuda.so`` (header ``include/lightship_cuda.h``)
built from ``lightship_b200/csrc``.  This Python package binds it with ctypes:

* ``lightship_b200.backend`` mirrors LightShip's ``Backend`` trait
  (lightship-core/src/backend/backend.rs:128-163): compile_operator / execute / allocate /
  deallocate / synchronize, over host or device tensors.
* ``lightship_b200.ops`` exposes the kernel-level entry points on torch device tensors.

There is no CPU fallback: importing an operator module without the built library raises.
"""
__version__ = "0.1.0"
