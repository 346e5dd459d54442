// noalloc.cu -- device scratch that is never allocated at run time.
//
// The fused QKV GEMM reads the RoPE (cos, sin) table of the sequence from
// global memory; the table is scratch, made by k_rope_table just before the
// GEMM.  exn_test_qkv keeps it in step buffers that it grows with cudaMalloc.
// exn_qkv_noalloc (dit.cpp) instead uses the fixed array below, which the CUDA
// runtime places in device memory when it loads this library's module on a
// device, and which every device that loaded the module holds until the
// process exits.  Host code never names the array: on the host its name is a
// stand-in, not a device address, so the address is looked up once per device
// with cudaGetSymbolAddress and handed to the kernels as a plain pointer.
#include <mutex>

#include "exn_internal.h"

namespace exn {

// rows x 64 (cos, sin) pairs: 8704 rows x 512 bytes = 4.25 MiB
static __device__ __align__(256) float2 g_rope_scratch[kNoAllocMaxRows * 64];

static constexpr int kMaxDevices = 64;

int noalloc_rope_scratch(int device, float2** table) {
  static std::mutex mu;
  static float2* addr[kMaxDevices] = {};
  if (device < 0 || device >= kMaxDevices || !table) return -1;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[device]) {
    // the caller made DEVICE current: the symbol resolves to that device's copy
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_rope_scratch);
    if (e != cudaSuccess) return static_cast<int>(e);
    addr[device] = static_cast<float2*>(p);
  }
  *table = addr[device];
  return 0;
}

}  // namespace exn
