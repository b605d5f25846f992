// pkv_lib.cu -- single translation unit of libprismkv_b200.so (the kernels
// share the device error word without relocatable device code).
#include "pkv_codec.cu"
#include "pkv_encode_tc.cu"
#include "pkv_attn.cu"
#include "pkv_scores.cu"
#include "pkv_api.cu"
#include "pkv_noalloc.cu"
