// nd_kv_f32.cu - append/attend kernels for float KV caches.
#include "nd_kv_inst.cuh"
ND_DEFINE_KV(f32, float)
