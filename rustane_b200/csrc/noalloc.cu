// Allocation-free variant of the attention backward pass.
//
// rt_kernel_attention_bwd needs a scratch vector (rowsum(dO * O), one float per
// batch x head x position) that its caller allocates.  Some callers cannot call
// cudaMalloc at the point where they run the backward pass: a process whose
// device memory is owned by another allocator (for example a framework's
// caching allocator that has already reserved nearly all HBM, so a raw
// cudaMalloc would fail or fragment it), or a step loop that must not pay the
// implicit device synchronisation cudaMalloc / cudaFree can trigger.  For them,
// rt_kernel_attention_bwd_noalloc takes the scratch from a fixed array compiled
// into this library instead, and allocates nothing.
//
// The array holds kNoAllocDvecMax floats (2 MiB); every GPU that loads the
// library keeps it for the life of the process.  Calls with
// batch * heads * seq > kNoAllocDvecMax are rejected with RT_ERR_SHAPE.
//
// All calls share the one array and it keeps the previous call's contents.
// Nothing in it needs to start at zero: the first kernel of the backward pass
// writes every element that the later kernels read.  Two calls whose work
// overlaps on the GPU (for example on two streams) race on the array; callers
// must order them (one stream, or events).
#include <mutex>

#include "attention.h"
#include "rustane_cuda.h"

namespace {

constexpr int64_t kNoAllocDvecMax = int64_t(1) << 19;  // floats: 2 MiB
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_dvec[kNoAllocDvecMax];

std::mutex g_mu;
float* g_dvec_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device.  The host-side
// name g_noalloc_dvec is only a handle for the symbol, not a device pointer,
// so the address is looked up once per device (with that device current) and
// cached.  This lookup happens inside the first call on each device; that
// first call should come before any stream capture on that device.
int dvec_on_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RT_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return RT_ERR_ARG;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_dvec_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_dvec);
    if (e != cudaSuccess || p == nullptr) return RT_ERR_CUDA;
    g_dvec_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_dvec_ptr[dev];
  return RT_OK;
}

}  // namespace

extern "C" {

RT_API int rt_kernel_attention_bwd_noalloc(const void* qkv, const void* out, const float* lse2, const void* dout,
                                           void* dqkv, const float* rope_cos_b, const float* rope_sin_b, int batch,
                                           int seq, int heads, void* stream) {
  if (!qkv || !out || !lse2 || !dout || !dqkv || !rope_cos_b || !rope_sin_b) return RT_ERR_ARG;
  if (batch <= 0 || seq <= 0 || heads <= 0) return RT_ERR_ARG;
  if (int64_t(batch) * heads * seq > kNoAllocDvecMax) return RT_ERR_SHAPE;
  float* dvec = nullptr;
  const int rc = dvec_on_current_device(&dvec);
  if (rc != RT_OK) return rc;
  rt::AttnArgs a;
  a.batch = batch;
  a.S = seq;
  a.heads = heads;
  a.hd = 128;
  a.D = heads * 128;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.ldq = 3 * a.D;
  a.out = const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(out));
  a.ldo = a.D;
  a.lse2 = const_cast<float*>(lse2);
  a.dout = static_cast<const __nv_bfloat16*>(dout);
  a.lddo = a.D;
  a.dvec = dvec;
  a.dqkv = static_cast<__nv_bfloat16*>(dqkv);
  a.lddq = 3 * a.D;
  a.rope_cos_b = rope_cos_b;
  a.rope_sin_b = rope_sin_b;
  const int lr = rt::attn_backward(a, static_cast<cudaStream_t>(stream));
  return lr == 0 ? RT_OK : (lr == -1 ? RT_ERR_SHAPE : RT_ERR_CUDA);
}

}  // extern "C"
