// b3_internal.h — shared declarations of the CUDA library (not part of the ABI).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "../../include/bark3_b200.h"

namespace b3 {

// Default wall-time bound of a device-side wait (2 s: orders of magnitude
// above any legitimate wait in these kernels).
constexpr unsigned long long kDefaultWaitNs = 2000000000ull;

// ── errors: every ABI call returns 0 or a negative B3_E* code and leaves a
// message in the calling thread's last-error slot.
int set_error(int code, const char* fmt, ...);
int set_cuda_error(const char* what, cudaError_t e);
void clear_error();

// Runs a set-up step once per device (the device current at the call) for
// one call site.  Kernel attributes such as the dynamic shared-memory limit
// belong to a device, so a process that drives several GPUs (one host thread
// per context) must set them on each; concurrent first calls from several
// threads run the step once per device.  Returns 0 or the step's error.
class PerDeviceOnce {
public:
    template <typename F>
    int run(F&& step) {
        int dev = 0;
        const cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return set_cuda_error("cudaGetDevice", e);
        if (dev < 0 || dev >= 64) return set_error(B3_EINVAL, "device ordinal %d is beyond 63", dev);
        const uint64_t bit = 1ull << dev;
        if (done_.load(std::memory_order_acquire) & bit) return 0;
        std::lock_guard<std::mutex> lock(mu_);
        if (done_.load(std::memory_order_relaxed) & bit) return 0;
        const int rc = step();
        if (rc == 0) done_.fetch_or(bit, std::memory_order_release);
        return rc;
    }

private:
    std::atomic<uint64_t> done_{0};
    std::mutex mu_;
};

// cudaFuncSetAttribute(kernel, MaxDynamicSharedMemorySize, bytes) once per
// device for the given call site's PerDeviceOnce.
template <typename K>
int set_smem_limit_once(PerDeviceOnce& once, K kernel, int bytes, const char* what) {
    return once.run([&]() {
        const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        return e == cudaSuccess ? 0 : set_cuda_error(what, e);
    });
}

// Streaming multiprocessors of the current device (cached per device).
int device_sms();

// ── K1 GEMM ──
enum GemmEpi {
    EPI_F32 = 0,       // out_f32 = acc (+ bias)
    EPI_RESID = 1,     // out_f32 += alpha * acc
    EPI_F16 = 2,       // out_f16 = f16(acc (+ bias))
    EPI_SILU_F16 = 3,  // out_f16 = f16(silu(acc (+ bias)))
    EPI_GLU_F16 = 4,   // out_f16[:, i] = f16(acc[2i] * sigmoid(acc[2i+1]))
    EPI_QKV = 5,       // out_f16 row = [q + bias_u | q + bias_v | k | v]
    EPI_RELU_F16 = 6,  // out_f16 = f16(max(acc + bias, 0))
};

struct GemmParams {
    int M, N, K;
    int ldo;                  // row stride of the output, in elements
    float alpha;              // residual scale (EPI_RESID)
    const float* bias;        // [N] or null
    const float* bias_u;      // [1024] (EPI_QKV)
    const float* bias_v;      // [1024] (EPI_QKV)
    const uint16_t* lut;      // [N][16] f16 bits (LUT4 weights)
    float* out_f32;
    __half* out_f16;
    // split-K (EPI_F32 only): the K range is cut into ksplit equal parts and
    // part s writes its partial sums to rows
    // [s * gemm_split_rows(M), s * gemm_split_rows(M) + M) of out_f32 (the
    // bias goes into part 0 only); the consumer adds the parts in order.
    // 0 or 1 = no split.
    int ksplit;
    int tiles;                // 0 = by size, 1 = 128 x 64 tiles, 2 = 256 x 128 tiles, 3 = 256 x 256 on CTA pairs
    int pdl;                  // launch with programmatic stream serialization (single-CTA tiles)
};

struct GemmOp {
    CUtensorMap map_a;
    CUtensorMap map_b;
    GemmParams p;
    bool lut;
    int epi;
};

// TMA 2D map over a row-major matrix; dtype kMapU8 / kMapF16 / kMapF32.
constexpr int kMapU8 = 0, kMapF16 = 1, kMapF32 = 2;
int make_map_2d(CUtensorMap* map, const void* base, int dtype, uint64_t inner, uint64_t outer,
                uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, bool swizzle128);
// TMA 3D map: dims[0] innermost (contiguous), stride_bytes[i] between
// consecutive indices of dims[i + 1].
int make_map_3d(CUtensorMap* map, const void* base, int dtype, const uint64_t dims[3], const uint64_t stride_bytes[2],
                const uint32_t box[3], bool swizzle128);
int gemm_make_a_map(CUtensorMap* map, const __half* a, int M, int K, int lda);
int gemm_make_b_map(CUtensorMap* map, const void* w, bool lut, int N, int K);
int gemm_validate(const GemmParams& p, bool lut);
int gemm_launch(const GemmOp& op, cudaStream_t st);
// Rows of one split-K part in the output (M rounded up to the 256-row tile).
__host__ __device__ inline int gemm_split_rows(int M) { return (M + 255) / 256 * 256; }
// Split-K plan for a small-M GEMM: tile shape (1 = 128 x 64, 2 = 256 x 128)
// and number of K parts that keep every SM busy with the fewest bytes each.
void gemm_plan_split(int M, int N, int K, bool lut, int num_sms, int max_parts, int* tiles, int* ksplit);
int gemm_take_dev_error(cudaStream_t st, unsigned int* out);

}  // namespace b3
