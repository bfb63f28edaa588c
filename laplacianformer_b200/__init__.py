"""B200 (sm_100a) implementation of LaplacianFormer's two custom operators.

* ``Laplace_subtraction_cuda`` (repository root) — drop-in PyTorch extension
  with the reference's module, operator names and signatures.
* :mod:`laplacianformer_b200.capi` — ctypes binding of the C ABI
  (include/laplacian_b200.h, liblfb200.so).
* :mod:`laplacianformer_b200.ops` — autograd functions.
* :mod:`laplacianformer_b200.sharding` — B*H sharding over ranks.
* :mod:`laplacianformer_b200.workloads` — seeded benchmark inputs.
"""
__version__ = "0.1.0"
