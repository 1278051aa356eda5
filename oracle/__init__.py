"""CPU oracle for the B200 PP-OCR layer path. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import, call, link or run anything in this package, and only as the
checker or the timed CPU baseline -- never as the product path.

Contents
  layers.py   torch-CPU float32 restatement of every layer operator with the
              reference's fp16 storage/rounding points
  models.py   runs a generated graph's layer list through layers.py
  ctc_oracle.c  plain-C restatement of the CTC head on the host: row argmax
              (ties -> lowest id) + softmax-max over fp16 logits, and the
              greedy collapse (repeat-then-blank, mean kept score)
  ref_*.c*/Makefile  shims that compile the reference's own sources
              (ctc_decode.cpp, classifier.cu, spatial_kernels.cuh) where they
              lie into oracle/_ref/ to pin the restatement

Parity pinning:
  * CTC collapse: pinned to the reference test's golden vectors
    (native/tests/tools/ctc_smoke.cpp:21-38) and to the compiled reference
    ctc_decode.cpp on seeded inputs.
  * classifier argmax/prob and depthwise/pool kernels: pinned on the GPU box
    against the reference's own classifier.cu and spatial_kernels.cuh,
    compiled from source into oracle/_ref.
  * dense convolutions, GEMMs, attention, LayerNorm: restated from
    native/src/compiled/runtime.cuh; the reference runs these through cuDNN /
    cuBLAS (closed libraries) and its runtime needs them to build, so these
    restatements are parity-unpinned beyond the source reading.
"""
