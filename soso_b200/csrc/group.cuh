// group.cuh -- tensor-parallel groups of GPUs of one node: the exchange areas through
// which a kernel hands its share of a result to every rank of the group.
//
// The reference runs on one device (its multi-machine mode is a TCP layer pipeline,
// crates/soso-llm-core/src/pipeline.rs); the sharded decode here is new.  One process
// drives one GPU; every rank allocates one exchange area and the ranks swap CUDA IPC
// handles to it (through whatever host channel they share: torch.distributed in
// soso_b200), so each rank can store into every peer's area over NVLink.
//
// A publishing kernel (a matvec whose rows are this rank's share of a sum, or the
// argmax of this rank's slice of the vocabulary) stores its values into a data slot of
// every rank's area, fences, and adds 1 per CTA to that area's counter of (exchange
// point k, source rank).  Tensor-parallel partial sums go to slot [rank]; the outputs
// of routed experts (expert parallelism) go to slot [choice], the expert's position in
// the token's top-k, whichever rank owns the expert.  A consuming kernel waits, with a
// bounded spin, until every source's counter has reached epoch * (CTAs per publisher)
// and then sums the slots in slot order with its weights (a fixed order: every rank
// forms bit-identical sums).
// Exchange points are numbered within a token; data slots alternate by the parity of
// k, which is enough because no rank can publish exchange k + 2 before every rank has
// consumed exchange k (it needs their k + 1 shares first).  Counters only grow: the
// epoch (tokens started on this group, device memory) scales their targets, so nothing
// is ever reset between tokens.
#pragma once
#include "common.cuh"

namespace sb {
namespace grp {

constexpr int MAXG = 8;          // ranks
constexpr int DSL = 24;          // data slots per parity (ranks, or top-k choices + a shared expert)
constexpr int XW = 16384;        // floats per data slot (hidden size at most)
constexpr int NX = 512;          // exchange points per token
constexpr unsigned WAIT_LIMIT = 1u << 26;

// [data: 2][DSL][XW] f32 | [arg: MAXG][2] u32 | [cnt: NX][MAXG] u32
constexpr size_t DATA_BYTES = (size_t)2 * DSL * XW * 4;
constexpr size_t ARG_OFF = DATA_BYTES;
constexpr size_t CNT_OFF = ARG_OFF + (size_t)MAXG * 8;
constexpr size_t AREA_BYTES = CNT_OFF + (size_t)NX * MAXG * 4;

__host__ __device__ inline float *data_slot(void *area, int k, int slot)
{
    return reinterpret_cast<float *>(area) + ((size_t)(k & 1) * DSL + slot) * XW;
}
__host__ __device__ inline unsigned *arg_slot(void *area, int src)
{
    return reinterpret_cast<unsigned *>(reinterpret_cast<char *>(area) + ARG_OFF) + 2 * src;
}
__host__ __device__ inline unsigned *cnt_slot(void *area, int k, int src)
{
    return reinterpret_cast<unsigned *>(reinterpret_cast<char *>(area) + CNT_OFF) + (size_t)k * MAXG + src;
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p)
{
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait until cnt[s] >= target for s < n; false (and the device error word set)
// if the limit ran out.
__device__ inline bool wait_counts(const unsigned *cnt, int n, unsigned target, unsigned limit = WAIT_LIMIT)
{
    for (int s = 0; s < n; s++) {
        unsigned it = 0;
        while (ld_acquire_sys(cnt + s) < target) {
            if (++it > limit) {
                set_dev_error(0x91u);
                return false;
            }
            __nanosleep(100);
        }
    }
    return true;
}

// Where a kernel publishes its share of exchange point k.
struct Pub {
    float *dst[MAXG];       // a data slot of every rank's area (matrix i of a batch adds its pub_off)
    unsigned *cnt[MAXG];    // counter (k, rank) of every rank's area
    int n;                  // ranks (0: not publishing)
};

// What a kernel waits for before reading exchange point k from its own area.
struct Wait {
    const unsigned *cnt;    // counters (k, 0..n-1) of the own area
    const unsigned *epoch;  // device epoch (tokens started)
    int n;                  // ranks (0: nothing to wait for)
    int per;                // counter increments per source per token (publisher CTAs)
};

// The consuming side of an exchange point on its own (one thread): the same bounded wait,
// with the caller's spin limit; ok = 1 when every counter reached the target.
__global__ void exchange_wait_kernel(const unsigned *cnt, int n, unsigned target, unsigned limit, int *ok)
{
    if (threadIdx.x == 0) *ok = wait_counts(cnt, n, target, limit) ? 1 : 0;
}

}  // namespace grp
}  // namespace sb

// Wait (bounded) for n exchange counters (device memory) to reach target, as a consuming
// kernel does before it reads an exchange point; ok (device int) gets 1, or 0 when `limit`
// spins ran out -- and then the device error word holds 0x91.  A wait that nothing
// satisfies costs about limit x 100 ns.
extern "C" int sbk_exchange_wait(const unsigned *cnt, int n, unsigned target, unsigned limit, int *ok, void *stream)
{
    if (!cnt || !ok || n < 1 || n > sb::grp::MAXG || !limit || limit > sb::grp::WAIT_LIMIT) return -1;
    sb::grp::exchange_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(cnt, n, target, limit, ok);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

struct sb_group {
    int rank = 0, world = 1;
    void *area = nullptr;                       // own exchange area (cudaMalloc)
    void *peer[sb::grp::MAXG] = {};             // every rank's area as mapped here (peer[rank] = area)
    unsigned *epoch = nullptr;                  // device: tokens started on this group
    float *ones = nullptr;                      // device: MAXG x 1.0f (weights of the rank sum)
    bool opened = false;
};
