"""B200-native W8A8 / W4A8 quantized-conv inference engine (sm_100a).

Host side of the engine: a thin ctypes mirror of the reference's
``Model`` / ``load_ptqc`` / ``Int8Engine`` interface over the C-ABI library
``libptq8.so`` (declared in ``include/ptq8.h``).
"""
