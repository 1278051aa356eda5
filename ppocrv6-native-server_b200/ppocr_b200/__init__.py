"""Host side of the B200 PP-OCR layer path: build, model catalog, ctypes
bindings of the C-ABI libraries. The compute path is the sm_100a code in
../csrc; nothing here computes on the CPU."""
