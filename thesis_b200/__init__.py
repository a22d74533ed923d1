"""B200-native packed LayerSkip-Llama draft/verify step: a C-ABI library of sm_100a kernels
(``thesis_b200/_lib/libeesd.so``, declared in ``include/eesd.h``) behind the reference's
``DecodeEngine`` / method-registry interface."""
