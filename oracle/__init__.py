"""CPU oracle for the nvmoe_b200 hot path — TEST INFRASTRUCTURE ONLY.

This package restates the reference algorithm on the CPU so the CUDA path can be checked
against it.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
may import it; the product (nvmoe_b200/) never does.

Parity pins (what the restatement itself is checked against):
  - dequant: gguf-py 0.19.0 (the installed copy of ggml's reference dequantizers; Q2_K,
    IQ2_XXS, and NVFP4 through the FTW -> block_nvfp4 packing of
    scripts/convert_ftw_to_gguf.py:46-70) — tests/test_oracle_pins.py;
  - host tier (SLRU): the reference's own scripts/segmented_host_lru.hpp compiled into
    oracle/_ref by oracle/Makefile, its 7 known-answer tests (test_segmented_host_lru.cpp),
    and traces of the reference's Python SegmentedHostLru committed under tests/golden/;
  - remap / eval_cb GPU tier: restated in C (oracle/remap_lru.c) from
    scripts/moe_cache_probe.cpp:627-753,955-970; the reference engine needs ggml + liburing +
    CUDA and cannot be built here, so this row is pinned by the reference's invariants
    (shrunk + remapped ids == full, test_mul_mat_id_shrink.cpp) and by the committed traces;
  - FFN arithmetic: no reference implementation exists in the source tree (FreeToken's Marlin
    kernel and ggml mul_mat_id are absent) — parity unpinned; the oracle is the fp32
    restatement of y = sum_j w_j * down(silu(gate x) * up x).
"""
