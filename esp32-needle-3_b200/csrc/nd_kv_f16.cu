// nd_kv_f16.cu - append/attend kernels for __half KV caches.
#include "nd_kv_inst.cuh"
ND_DEFINE_KV(f16, __half)
