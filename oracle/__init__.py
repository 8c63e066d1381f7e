"""TEST INFRASTRUCTURE ONLY: the CPU oracle of the paged KV cache data path.

pkv_oracle.c restates the reference's CpuBackend (cpu.rs) and the trait's
default batch methods (backend.rs); host_ref.py restates BlockAllocator,
BlockTable and Scheduler. Only tests/, the smoke check and the benchmark's
CPU-baseline leg use this package, and only as the checker.
"""
