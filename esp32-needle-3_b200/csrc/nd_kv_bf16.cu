// nd_kv_bf16.cu - append/attend kernels for __nv_bfloat16 KV caches.
#include "nd_kv_inst.cuh"
ND_DEFINE_KV(bf16, __nv_bfloat16)
