"""Checkpoint formats and seeded synthetic workloads of the decoder hot path.

Library-free on purpose: nothing here loads libg4b200.so, so the CPU-only users (the
reference arm of bench.py, the CPU oracle tests) can build the same inputs as the GPU
path without mapping the product library.

- `quant`: the NVFP4 / FP8 storage formats of the reference checkpoint
  (src/host/load.rs:10-191) and the seeded N(0, sigma) workloads built on them.
- `tp`: the tensor-parallel cut of those tensors that a rank's context expects.
"""
