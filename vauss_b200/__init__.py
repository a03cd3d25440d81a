"""vauss_b200: the Gaussian-splat training step on B200 (sm_100a).

Kernels live in ``csrc/`` behind the C ABI of ``include/vauss_b200.h``
(built in-tree into ``_lib/libvauss_b200.so``); ``ops`` wraps each entry
point for torch tensors, ``trainer`` and ``view_parallel`` are the training
step on one and on several GPUs, ``refine``, ``dataset`` and ``checkpoint``
are densification, the staged ground-truth feed and PLY / moment I/O.
"""
