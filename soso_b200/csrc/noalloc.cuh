// noalloc.cuh -- a Q4_K matvec entry point that allocates no device memory.
//
// Some callers cannot call cudaMalloc: code that runs inside a memory pool they
// do not own (a host engine that budgets every byte of device memory up front),
// code that may run while another thread is capturing a CUDA graph in global
// capture mode (where an allocation call invalidates that capture), and
// latency-critical paths that must not hit the driver's allocator.  For them,
// sbk_matvec_q4k_noalloc runs the same kernel as sbk_matvec(SB_DTYPE_Q4_K, ...)
// but takes its scratch memory (the per-group counters and the per-CTA partial
// sums of rows split between CTAs) from the fixed array below instead of a
// lazily allocated workspace.
//
// The array lives in the library image: every GPU that loads the library holds
// its NOALLOC_SCRATCH_BYTES until the process exits.  All calls on a device share
// it and it keeps the last call's contents, so calls whose kernels overlap on the
// GPU (two streams, or two threads) race on it; serialise them.  The counters
// must start at zero: each call clears them with cudaMemsetAsync (no allocation).
//
// Host code cannot use the array's name as a device address (it names a host
// stand-in), so the first call on each device looks the address up with
// cudaGetSymbolAddress while that device is current, and later calls reuse it.
// Make that first call before any stream capture.
#pragma once
#include "tc_mmv.cuh"

namespace sb {
namespace noalloc {

constexpr int MAX_GROUPS = 16384;  // rows <= 262144
constexpr int MAX_CTAS = 256;
constexpr size_t CNT_BYTES = (size_t)MAX_GROUPS * 4;
constexpr size_t PART_BYTES = (size_t)MAX_CTAS * 2 * 16 * 4;
constexpr size_t NOALLOC_SCRATCH_BYTES = CNT_BYTES + PART_BYTES;  // 96 KiB

static __device__ __align__(256) unsigned char g_scratch[NOALLOC_SCRATCH_BYTES];

// Device address of g_scratch on the current device, looked up once per device.
inline int scratch_ptr(void **out)
{
    static void *ptrs[64];
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -3;
    std::lock_guard<std::mutex> lk(mu);
    if (!ptrs[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || !p) return -3;
        ptrs[dev] = p;
    }
    *out = ptrs[dev];
    return 0;
}

}  // namespace noalloc
}  // namespace sb

extern "C" int sbk_matvec_q4k_noalloc(const void *w, size_t rows, size_t cols, const float *x, float *y,
                                      void *stream)
{
    using namespace sb;
    if (!w || !x || !y || rows == 0) return -1;
    if (((uintptr_t)w & 15) || ((uintptr_t)x & 15)) return -2;
    if (cols == 0 || cols % 256 || cols > (size_t)tcmv::Q4K::MAX_COLS) return -1;
    // the fixed scratch bounds the shape: one counter per 16 rows
    if ((rows + 15) / 16 > (size_t)noalloc::MAX_GROUPS) return -8;
    const int grid = num_sms_cached();
    if (grid > noalloc::MAX_CTAS) return -8;
    const tcmv::MatOp op{w, (int)rows, (int)cols, x, y};
    if (!tcmv::fits<tcmv::Q4K>(&op, 1, grid)) return -5;
    void *scratch = nullptr;
    if (noalloc::scratch_ptr(&scratch)) return -3;
    cudaStream_t s = (cudaStream_t)stream;
    // counters must start at zero (a call that failed midway may have left some set)
    if (cudaMemsetAsync(scratch, 0, (rows + 15) / 16 * 4, s) != cudaSuccess) return -4;
    tcmv::Ws wsd;
    wsd.cnt = reinterpret_cast<unsigned *>(scratch);
    wsd.part = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(scratch) + noalloc::CNT_BYTES);
    return tcmv::launch_batch_ws<tcmv::Q4K>(&op, 1, wsd, noalloc::MAX_GROUPS, grid, 0, s);
}
