"""TEST INFRASTRUCTURE ONLY -- the CPU oracle of the grouped multi-LoRA apply.

CPU restatements of the reference's algorithm for the apply path, used as the
checker by tests/, by __graft_entry__.smoke() and by the cpu_baseline /
--impl reference legs of bench.py. Nothing in the product package imports it.

  seg.py    numpy restatement of the segment-table builders
            (build_seg_bounds_kernel, csrc/kernels/warp_pipe_r32.cu:461-512;
             build_segment_table, csrc/dispatch/segment_builder.cpp:5-50)
  apply.py  torch fp32 restatement of the apply math
            (tests/correctness/reference_bgmv.py:4-18,
             tests/correctness/test_add_lora_packed.py:35-45)
  ref_shim.cu + build_ref.sh
            build oracle/_ref/libwpref.so from the reference's own CUDA
            kernels, so GPU tests can check against the reference itself.

Pinning: tests/golden/ holds fixtures made by the reference's own Python
functions (tests/golden/make_golden.py) and by the reference's own
build_seg_bounds kernel run on a B200 (tests/golden/make_ref_seg_golden.py).
"""
