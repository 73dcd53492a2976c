"""B200 (sm_100a) Gaussian-field weight-delta renderer for GUASS adapters.

Modules (import them directly; this package imports nothing eagerly):

* ``guass_b200.cuda_field`` -- drop-in for ``gaussian_peft.cuda_field``
  (extension object, autograd runtime, ``install()`` / ``uninstall()``).
* ``guass_b200.batched`` -- ``FieldBatch``: up to 192 fields per launch set.
* ``guass_b200.adapters`` -- ``BatchedAdapters`` / ``ModelRenderer`` (one
  render per step or per model forward), ``CheckpointFields``, data-parallel
  gradient all-reduce, adapter checkpoint entries.
* ``guass_b200.partition`` -- layer-partitioned multi-GPU render (NCCL,
  NVLink multicast, or the render storing through the multicast address).
* ``guass_b200.stats`` -- densify statistics in one launch.
* ``guass_b200.sd15`` -- SD1.5-shaped UNet training workload.
* ``guass_b200.synthetic`` -- seeded workloads of the benchmark configs.

The kernels live in ``libgfield.so`` (C ABI: ``include/gfield.h``), loaded
by ``guass_b200._lib``; there is no fallback implementation.
"""
