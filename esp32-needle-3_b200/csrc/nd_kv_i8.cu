// nd_kv_i8.cu - append/attend kernels for int8_t KV caches.
#include "nd_kv_inst.cuh"
ND_DEFINE_KV(i8, int8_t)
