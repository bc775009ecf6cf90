// noalloc.cu — b3_linear_lut4_noalloc: the single 4-bit linear without any
// device allocation.
//
// b3_linear_lut4 stages an f16 copy of the activations in context-owned
// device memory that it grows with cudaMalloc on demand.  Some callers cannot
// have that: latency-critical threads (a real-time audio host feeding the
// encoder chunk by chunk) must not block in cudaMalloc / cudaFree, which can
// synchronise the whole device, and hosts that account for every byte of GPU
// memory through their own pool cannot let a library allocate behind their
// back.  This entry point takes only caller-owned device buffers and stages
// the f16 activations in a fixed scratch array that lives in this file.
//
// The scratch is a file-scope __device__ array: every GPU that loads this
// library holds it (8 MiB) until the process exits.  In host code its name is
// only a host-side stand-in, so the device address is looked up once per
// device with cudaGetSymbolAddress, with that device current, on the first
// call on that device; make that first call before any stream capture.  All
// calls share the one array and it keeps the previous call's contents; the
// f32 -> f16 pass rewrites every element the GEMM then reads (rows past m are
// never read: the TMA map stops at m and fills zeros), so nothing has to be
// cleared between calls.  Calls whose work overlaps on the GPU (different
// streams, or different host threads on one device) race on the scratch.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "b3_internal.h"
#include "b3_kernels.h"

namespace b3 {
namespace {

// Largest m * k the scratch holds: 4 Mi f16 values (8 MiB), e.g. 4096 x 1024.
constexpr int64_t kNoallocMaxElems = 4ll << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) __half g_noalloc_a16[kNoallocMaxElems];

std::mutex g_noalloc_mu;
__half* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch on the current device (looked up once).
int noalloc_scratch(__half** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_cuda_error("cudaGetDevice", e);
    if (dev < 0 || dev >= kMaxDevices) return set_error(B3_EINVAL, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_a16);
        if (e != cudaSuccess) return set_cuda_error("cudaGetSymbolAddress(scratch)", e);
        g_noalloc_ptr[dev] = static_cast<__half*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return 0;
}

}  // namespace
}  // namespace b3

using namespace b3;

extern "C" int b3_linear_lut4_noalloc(const float* a, const uint8_t* codes, const uint16_t* lut16,
                                      const float* bias, float* c, int m, int n, int k, void* stream) {
    if (!a || !codes || !lut16 || !c) return set_error(B3_EINVAL, "null buffer");
    if (m <= 0 || n <= 0 || k <= 0 || k % 64 || n % 128)
        return set_error(B3_EINVAL, "linear shape m=%d n=%d k=%d (need k %% 64 == 0, n %% 128 == 0)", m, n, k);
    if (static_cast<int64_t>(m) * k > kNoallocMaxElems)
        return set_error(B3_EINVAL, "m * k = %lld exceeds the allocation-free scratch (%lld values, 8 MiB)",
                         static_cast<long long>(m) * k, static_cast<long long>(kNoallocMaxElems));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    __half* a16 = nullptr;
    int rc = noalloc_scratch(&a16);
    if (rc) return rc;
    rc = launch_f32_to_f16(a, a16, static_cast<int64_t>(m) * k, st);
    if (rc) return rc;
    GemmOp op;
    rc = gemm_make_a_map(&op.map_a, a16, m, k, k);
    if (rc) return rc;
    rc = gemm_make_b_map(&op.map_b, codes, true, n, k);
    if (rc) return rc;
    op.p = GemmParams{};
    op.p.M = m;
    op.p.N = n;
    op.p.K = k;
    op.p.ldo = n;
    op.p.bias = bias;
    op.p.lut = lut16;
    op.p.out_f32 = c;
    op.lut = true;
    op.epi = EPI_F32;
    return gemm_launch(op, st);
}
