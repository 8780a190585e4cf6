// dispatch.cuh -- the GpuDispatch surface (sb_*): host buffers in, host
// buffers out, weights resident per key.
//
// Mirrors CudaGpu (crates/soso-llm-api/src/cuda.rs): weights are uploaded on
// first sight and kept under their stable key (`pesos`, cuda.rs:290); a failed
// upload is remembered and not retried (cuda.rs:2364-2376); the device is made
// current on every call (cuda.rs:2362); shapes a kernel does not take are
// declined with 0 rather than failed (crates/soso-llm-api/tests/cuda_matvec.rs
// :275-282).  Unlike the reference there is no silent fallback in here: a
// declined op returns 0 and the caller decides.
#pragma once
#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "group.cuh"
#include "sosob200.h"

extern "C" int sbk_matvec(uint8_t dtype, const void *w, size_t rows, size_t cols, const float *x, float *y,
                          int pdl, void *stream);
extern "C" int sbk_rmsnorm(const float *x, const float *res, float *h_out, const float *w, float *y, size_t rows,
                           size_t n, float eps, void *stream);
extern "C" int sbk_matvec_batch(uint8_t dtype, const sbk_mv_op *ops, size_t n, int pdl, void *stream);
extern "C" int sbk_q6k_pack(const void *src, size_t rows, size_t cols, void *dst, void *stream);
extern "C" int sbk_q80_pad(const void *src, size_t rows, size_t cols, void *dst, void *stream);

namespace {

thread_local std::string t_last_error;

int fail(const char *where, cudaError_t e)
{
    t_last_error = std::string(where) + ": " + cudaGetErrorString(e);
    return -1;
}

int fail(const std::string &msg)
{
    t_last_error = msg;
    return -1;
}

struct Resident {
    void *ptr = nullptr;
    size_t bytes = 0;
    uint8_t dtype = 0;      // as given (the reference's dtype)
    uint8_t dev_dtype = 0;  // as held on the device (Q6_K is repacked to Q6_K_P for matvecs)
    bool ok = false;
};

bool kernel_dtype(uint8_t d) { return d == SB_DTYPE_Q8_0 || d == SB_DTYPE_Q4_K || d == SB_DTYPE_Q6_K; }

}  // namespace

constexpr size_t PREFILL_MIN_TOKENS = 16;  // sb_matmul: from this many tokens on, the tcgen05 GEMM

struct sb_engine;                  // whole-token decode state (engine.cuh)
void sb_engine_free(sb_engine *e);
void sb_pf_free(void *p);          // its block-prefill state (prefill_engine.cuh)
// The host copies of a call between the caller's (pageable) buffers and the pinned staging
// buffer, spread over a few threads: one thread copies at ~10 GB/s, which for a batch of
// matvecs (1.5 MB of x and y for the configs[1] sweep) takes longer than the kernels.  The
// calling thread takes part 0 of the bytes, the workers the rest; workers spin for a short
// while after a job (calls tend to come back to back) and then sleep.
struct HostCopy {
    void *dst;
    const void *src;
    size_t n;
};

class CopyPool {
  public:
    explicit CopyPool(int workers)
    {
        for (int i = 0; i < workers; i++) th_.emplace_back([this, i] { loop(i + 1); });
    }
    ~CopyPool()
    {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_.store(true);
        }
        cv_.notify_all();
        for (auto &t : th_) t.join();
    }
    // All copies done when it returns.
    void run(const std::vector<HostCopy> &c)
    {
        size_t total = 0;
        for (const HostCopy &h : c) total += h.n;
        if (th_.empty() || total < (128u << 10)) {
            for (const HostCopy &h : c) memcpy(h.dst, h.src, h.n);
            return;
        }
        jobs_ = c.data(), njobs_ = c.size(), total_ = total;
        left_.store((int)th_.size(), std::memory_order_relaxed);
        {
            std::lock_guard<std::mutex> lk(mu_);
            gen_.fetch_add(1, std::memory_order_release);
        }
        cv_.notify_all();
        part(0);
        while (left_.load(std::memory_order_acquire) > 0) std::this_thread::yield();
    }

  private:
    // bytes [total * p / parts, total * (p + 1) / parts) of the copies, in list order
    void part(int p)
    {
        const size_t parts = th_.size() + 1, b0 = total_ * p / parts, b1 = total_ * (p + 1) / parts;
        size_t at = 0;
        for (size_t i = 0; i < njobs_ && at < b1; i++) {
            const HostCopy &h = jobs_[i];
            const size_t s = std::max(at, b0), e = std::min(at + h.n, b1);
            if (s < e) memcpy((char *)h.dst + (s - at), (const char *)h.src + (s - at), e - s);
            at += h.n;
        }
    }
    void loop(int id)
    {
        unsigned seen = 0;
        for (;;) {
            unsigned g = gen_.load(std::memory_order_acquire);
            for (int spin = 0; g == seen && spin < 4000 && !stop_.load(); spin++) {
                std::this_thread::yield();
                g = gen_.load(std::memory_order_acquire);
            }
            if (g == seen) {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return stop_.load() || gen_.load(std::memory_order_acquire) != seen; });
                if (stop_.load()) return;
                g = gen_.load(std::memory_order_acquire);
            }
            seen = g;
            part(id);
            left_.fetch_sub(1, std::memory_order_release);
        }
    }
    std::vector<std::thread> th_;
    std::mutex mu_;
    std::condition_variable cv_;
    std::atomic<unsigned> gen_{0};
    std::atomic<int> left_{0};
    std::atomic<bool> stop_{false};
    const HostCopy *jobs_ = nullptr;
    size_t njobs_ = 0, total_ = 0;
};

struct sb_ctx;
void sb_kv_mirror_free(const sb_ctx *c);  // KV mirrors of sb_attention_prefill (experts.cuh)
void sb_moe_free(const sb_ctx *c);        // MoE layers of sb_moe_layer (moe_layer.cuh)

struct sb_ctx {
    int device = 0;
    sb_engine *eng = nullptr;
    cudaStream_t stream = nullptr;
    std::mutex mu;
    std::unordered_map<std::string, Resident> weights;
    void *scratch = nullptr;  // device staging for x / out of host calls
    size_t scratch_bytes = 0;
    void *host_stage = nullptr;  // pinned mirror of scratch: one DMA each way per call
    size_t host_stage_bytes = 0;
    sb_stats stats = {};
    sb_group *grp = nullptr;  // tensor-parallel group (sb_group_create / sb_group_open)
    std::unique_ptr<CopyPool> pool;  // host copies of the calls (made at the first large one)

    void copy(const std::vector<HostCopy> &c)
    {
        if (!pool) {
            const unsigned hw = std::thread::hardware_concurrency();
            pool.reset(new CopyPool((int)std::min(3u, hw > 2 ? hw / 2 - 1 : 0u)));
        }
        pool->run(c);
    }

    int ensure_host_stage(size_t bytes)
    {
        if (bytes <= host_stage_bytes) return 0;
        // copies still queued may read or write the old buffer: let them finish first
        if (host_stage) cudaDeviceSynchronize(), cudaFreeHost(host_stage);
        host_stage = nullptr;
        host_stage_bytes = 0;
        size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
        cudaError_t e = cudaHostAlloc(&host_stage, want, cudaHostAllocPortable);
        if (e != cudaSuccess) return fail("cudaHostAlloc(stage)", e);
        host_stage_bytes = want;
        return 0;
    }

    int ensure_scratch(size_t bytes)
    {
        if (bytes <= scratch_bytes) return 0;
        if (scratch) cudaFree(scratch);
        scratch = nullptr;
        scratch_bytes = 0;
        size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
        cudaError_t e = cudaMalloc(&scratch, want);
        if (e != cudaSuccess) return fail("cudaMalloc(scratch)", e);
        scratch_bytes = want;
        return 0;
    }

    // 1 = resident, 0 = declined (remembered failure or shape), <0 = error.  Q6_K
    // matrices are repacked (SB_DTYPE_Q6_K_P) unless for_matvec is false (tables read
    // row by row, like the embedding, stay in the reference layout).
    int resident(const char *key, const sb_view *v, size_t rows, size_t cols, Resident **out,
                 bool for_matvec = true)
    {
        auto it = weights.find(key);
        if (it != weights.end()) {
            if (!it->second.ok) return 0;
            if (it->second.bytes != v->len || it->second.dtype != v->dtype)
                return fail(std::string("key '") + key + "' re-used with a different tensor");
            *out = &it->second;
            return 1;
        }
        Resident r;
        r.bytes = v->len;
        r.dtype = v->dtype;
        r.dev_dtype = v->dtype;
        const bool pack = for_matvec && v->dtype == SB_DTYPE_Q6_K && rows * cols == v->elems &&
                          sbk_row_bytes(SB_DTYPE_Q6_K_P, cols) != 0 && cols <= 12288;
        // Q8_0 is held with 16-byte-aligned rows (SB_DTYPE_Q8_0_R) for the tensor-core kernel
        // (a plain copy when the rows are aligned already), so one resident form serves all
        const bool pad = for_matvec && v->dtype == SB_DTYPE_Q8_0 && rows * cols == v->elems &&
                         sbk_row_bytes(SB_DTYPE_Q8_0_R, cols) != 0 && cols <= 16384;
        cudaError_t e;
        if (pad) {
            void *tmp = nullptr;
            e = cudaMalloc(&tmp, v->len);
            if (e == cudaSuccess) e = cudaMalloc(&r.ptr, sbk_row_bytes(SB_DTYPE_Q8_0_R, cols) * rows + 64);
            if (e == cudaSuccess) e = cudaMemcpy(tmp, v->bytes, v->len, cudaMemcpyHostToDevice);
            if (e == cudaSuccess && sbk_q80_pad(tmp, rows, cols, r.ptr, nullptr) != 0) e = cudaErrorLaunchFailure;
            if (e == cudaSuccess) e = cudaDeviceSynchronize();
            if (tmp) cudaFree(tmp);
            r.dev_dtype = SB_DTYPE_Q8_0_R;
        } else if (pack) {
            // upload, then repack into the resident buffer (+64 B: bulk reads round up to 16 B)
            void *tmp = nullptr;
            e = cudaMalloc(&tmp, v->len);
            if (e == cudaSuccess) e = cudaMalloc(&r.ptr, sbk_row_bytes(SB_DTYPE_Q6_K_P, cols) * rows + 64);
            if (e == cudaSuccess) e = cudaMemcpy(tmp, v->bytes, v->len, cudaMemcpyHostToDevice);
            if (e == cudaSuccess && sbk_q6k_pack(tmp, rows, cols, r.ptr, nullptr) != 0) e = cudaErrorLaunchFailure;
            if (e == cudaSuccess) e = cudaDeviceSynchronize();
            if (tmp) cudaFree(tmp);
            r.dev_dtype = SB_DTYPE_Q6_K_P;
        } else {
            // +64 B so vectorised/bulk reads that round a range up to 16 B stay inside the allocation
            e = cudaMalloc(&r.ptr, v->len + 64);
            if (e == cudaSuccess) e = cudaMemcpy(r.ptr, v->bytes, v->len, cudaMemcpyHostToDevice);
        }
        if (e != cudaSuccess) {
            if (r.ptr) cudaFree(r.ptr);
            r.ptr = nullptr;
            weights[key] = r;  // remembered: not retried
            cudaGetLastError();
            return 0;
        }
        r.ok = true;
        stats.bytes_up += v->len;
        auto res = weights.emplace(key, r);
        *out = &res.first->second;
        (void)rows;
        (void)cols;
        return 1;
    }
};

namespace {

// Shape/dtype admission shared by matvec/matmul: 1 ok, 0 decline.
int admit(const sb_view *w, size_t rows, size_t cols)
{
    if (!w || !w->bytes || !kernel_dtype(w->dtype)) return 0;
    if (w->elems != rows * cols || rows == 0) return 0;
    size_t rb = sbk_row_bytes(w->dtype, cols);
    if (!rb || w->len != rb * rows || cols > 65536) return 0;
    return 1;
}

uint64_t now_ns()
{
    return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

}  // namespace

extern "C" int sb_create(int device, sb_ctx **out)
{
    if (!out) return fail("sb_create: null out");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return fail("cudaGetDeviceCount", e);
    if (device < 0 || device >= n) return fail("sb_create: no such device");
    if ((e = cudaSetDevice(device)) != cudaSuccess) return fail("cudaSetDevice", e);
    cudaDeviceProp prop;
    if ((e = cudaGetDeviceProperties(&prop, device)) != cudaSuccess) return fail("cudaGetDeviceProperties", e);
    if (prop.major != 10) return fail("sb_create: kernels are built for sm_100a only");
    sb_ctx *c = new sb_ctx();
    c->device = device;
    if ((e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) != cudaSuccess) {
        delete c;
        return fail("cudaStreamCreate", e);
    }
    *out = c;
    return 0;
}

extern "C" void sb_destroy(sb_ctx *c)
{
    if (!c) return;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    if (c->eng) sb_engine_free(c->eng);
    sb_kv_mirror_free(c);
    sb_moe_free(c);
    for (auto &kv : c->weights)
        if (kv.second.ptr) cudaFree(kv.second.ptr);
    if (c->scratch) cudaFree(c->scratch);
    if (c->host_stage) cudaFreeHost(c->host_stage);
    if (c->grp) {
        for (int p = 0; p < c->grp->world; p++)
            if (p != c->grp->rank && c->grp->peer[p]) cudaIpcCloseMemHandle(c->grp->peer[p]);
        if (c->grp->area) cudaFree(c->grp->area);
        if (c->grp->epoch) cudaFree(c->grp->epoch);
        if (c->grp->ones) cudaFree(c->grp->ones);
        delete c->grp;
    }
    cudaStreamDestroy(c->stream);
    delete c;
}

extern "C" size_t sb_group_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int sb_group_create(sb_ctx *c, int rank, int world, void *handle_out)
{
    if (!c || !handle_out) return fail("null argument");
    if (world < 1 || world > sb::grp::MAXG || rank < 0 || rank >= world) return fail("sb_group_create: bad rank/world");
    std::lock_guard<std::mutex> lk(c->mu);
    if (c->grp) return fail("sb_group_create: the context already has a group");
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return fail("cudaSetDevice", e);
    sb_group *g = new sb_group();
    g->rank = rank, g->world = world;
    const float ones[sb::grp::MAXG] = {1, 1, 1, 1, 1, 1, 1, 1};
    const unsigned one = 1;
    if ((e = cudaMalloc(&g->area, sb::grp::AREA_BYTES)) == cudaSuccess &&
        (e = cudaMemset(g->area, 0, sb::grp::AREA_BYTES)) == cudaSuccess &&
        (e = cudaMalloc(&g->epoch, 64)) == cudaSuccess &&
        (e = cudaMemcpy(g->epoch, &one, 4, cudaMemcpyHostToDevice)) == cudaSuccess &&
        (e = cudaMalloc(&g->ones, sizeof(ones))) == cudaSuccess &&
        (e = cudaMemcpy(g->ones, ones, sizeof(ones), cudaMemcpyHostToDevice)) == cudaSuccess &&
        (e = cudaIpcGetMemHandle((cudaIpcMemHandle_t *)handle_out, g->area)) == cudaSuccess) {
        g->peer[rank] = g->area;
        c->grp = g;
        return 0;
    }
    if (g->area) cudaFree(g->area);
    if (g->epoch) cudaFree(g->epoch);
    if (g->ones) cudaFree(g->ones);
    delete g;
    return fail("sb_group_create", e);
}

extern "C" int sb_group_open(sb_ctx *c, const void *handles)
{
    if (!c || !handles) return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    sb_group *g = c->grp;
    if (!g) return fail("sb_group_open: no group (sb_group_create first)");
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return fail("cudaSetDevice", e);
    const cudaIpcMemHandle_t *h = (const cudaIpcMemHandle_t *)handles;
    for (int p = 0; p < g->world; p++) {
        if (p == g->rank || g->peer[p]) continue;
        if ((e = cudaIpcOpenMemHandle(&g->peer[p], h[p], cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess)
            return fail("cudaIpcOpenMemHandle", e);
    }
    g->opened = true;
    return 0;
}

extern "C" int sb_available(const sb_ctx *c) { return c ? 1 : 0; }

extern "C" int sb_dtype_supported(const sb_ctx *c, uint8_t dtype) { return c && kernel_dtype(dtype) ? 1 : 0; }

extern "C" size_t sb_resident_count(const sb_ctx *c)
{
    if (!c) return 0;
    size_t n = 0;
    for (auto &kv : c->weights) n += kv.second.ok ? 1 : 0;
    return n;
}

extern "C" int sb_get_stats(const sb_ctx *c, sb_stats *out)
{
    if (!c || !out) return -1;
    *out = c->stats;
    return 0;
}

extern "C" const char *sb_last_error(void) { return t_last_error.c_str(); }

// y (n x rows) = X (n x cols) . W^T ; n == 1 is the matvec.
static int run_matvecs(sb_ctx *c, const char *key, const sb_view *w, size_t rows, size_t cols, size_t n,
                       const float *x, float *out)
{
    if (!c) return fail("null context");
    if (!key || !x || !out) return fail("null argument");
    if (!admit(w, rows, cols) || n == 0) return 0;
    std::lock_guard<std::mutex> lk(c->mu);
    const uint64_t t0 = now_ns();
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return fail("cudaSetDevice", e);
    Resident *r = nullptr;
    int rc = c->resident(key, w, rows, cols, &r);
    if (rc <= 0) return rc;
    const size_t xb = n * cols * 4, yb = n * rows * 4, xoff = (xb + 255) & ~(size_t)255;
    const size_t yoff = xoff + ((yb + 255) & ~(size_t)255);
    // batches of tokens go to the tensor-core prefill GEMM (f16 operands: the precision of
    // the reference's own mma.sync prefill), single tokens to the matvec
    const bool gemm = n >= PREFILL_MIN_TOKENS && r->dev_dtype == SB_DTYPE_Q4_K;
    const size_t wsb = gemm ? sbk_matmul_ws_bytes(n, cols) : 0;
    if (c->ensure_scratch(yoff + wsb) || c->ensure_host_stage(xoff + yb)) return -1;
    float *dx = (float *)c->scratch, *dy = (float *)((char *)c->scratch + xoff);
    char *hs = (char *)c->host_stage;
    c->copy({HostCopy{hs, x, xb}});
    if ((e = cudaMemcpyAsync(dx, hs, xb, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(x)", e);
    if (gemm) {
        int k = sbk_matmul(r->dev_dtype, r->ptr, rows, cols, n, dx, dy, (char *)c->scratch + yoff, SBK_PREC_F16, 0,
                           c->stream);
        if (k) return fail("sbk_matmul launch failed (" + std::to_string(k) + ")");
        c->stats.launches += 2;
    } else {
        for (size_t t = 0; t < n; t++) {
            int k = sbk_matvec(r->dev_dtype, r->ptr, rows, cols, dx + t * cols, dy + t * rows, 0, c->stream);
            if (k) return fail("sbk_matvec launch failed (" + std::to_string(k) + ")");
            c->stats.launches++;
        }
    }
    if ((e = cudaMemcpyAsync(hs + xoff, dy, yb, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(out)", e);
    if ((e = cudaStreamSynchronize(c->stream)) != cudaSuccess) return fail("cudaStreamSynchronize", e);
    c->copy({HostCopy{out, hs + xoff, yb}});
    c->stats.bytes_up += xb;
    c->stats.bytes_down += yb;
    c->stats.total_ns += now_ns() - t0;
    return 1;
}

extern "C" int sb_matvec(sb_ctx *c, const char *key, const sb_view *w, size_t rows, size_t cols, const float *x,
                         float *out)
{
    return run_matvecs(c, key, w, rows, cols, 1, x, out);
}

extern "C" int sb_matmul(sb_ctx *c, const char *key, const sb_view *w, size_t rows, size_t cols, size_t n,
                         const float *x, float *out)
{
    return run_matvecs(c, key, w, rows, cols, n, x, out);
}

extern "C" int sb_matvec_batch(sb_ctx *c, sb_matvec_op *ops, size_t nops, uint8_t *done)
{
    if (!c) return fail("null context");
    if (!ops || !done) return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    const uint64_t t0 = now_ns();
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return fail("cudaSetDevice", e);
    // pass 1: residency + scratch layout
    std::vector<Resident *> res(nops, nullptr);
    std::vector<size_t> xo(nops), yo(nops);
    size_t xend = 0, yb = 0;
    for (size_t i = 0; i < nops; i++) {
        done[i] = 0;
        sb_matvec_op &op = ops[i];
        if (!op.key || !op.x || !op.out || !admit(op.view, op.rows, op.cols)) continue;
        int rc = c->resident(op.key, op.view, op.rows, op.cols, &res[i]);
        if (rc < 0) return rc;
        if (rc == 0) res[i] = nullptr;
        if (!res[i]) continue;
        xo[i] = xend;
        xend += (op.cols * 4 + 255) & ~(size_t)255;
        yo[i] = yb;
        yb += (op.rows * 4 + 255) & ~(size_t)255;
    }
    if (xend == 0) return 1;
    // [all x | all y], mirrored in pinned host memory: the inputs go up in one copy and
    // the outputs come down in one copy (a pageable copy per op costs far more than the op)
    if (c->ensure_scratch(xend + yb) || c->ensure_host_stage(xend + yb)) return -1;
    char *base = (char *)c->scratch, *hs = (char *)c->host_stage;
    std::vector<HostCopy> cp;
    for (size_t i = 0; i < nops; i++)
        if (res[i]) cp.push_back(HostCopy{hs + xo[i], ops[i].x, ops[i].cols * 4});
    c->copy(cp);
    if ((e = cudaMemcpyAsync(base, hs, xend, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(x)", e);
    // the kernels grouped by dtype (one launch per batch of Q4_K matrices), one wait
    std::vector<std::pair<uint8_t, std::vector<sbk_mv_op>>> by_dtype;
    for (size_t i = 0; i < nops; i++) {
        if (!res[i]) continue;
        sb_matvec_op &op = ops[i];
        yo[i] += xend;
        const uint8_t dt = res[i]->dev_dtype;
        size_t k = 0;
        while (k < by_dtype.size() && by_dtype[k].first != dt) k++;
        if (k == by_dtype.size()) by_dtype.push_back({dt, {}});
        by_dtype[k].second.push_back(sbk_mv_op{res[i]->ptr, op.rows, op.cols, (const float *)(base + xo[i]),
                                               (float *)(base + yo[i])});
        c->stats.bytes_up += op.cols * 4;
        c->stats.bytes_down += op.rows * 4;
    }
    for (auto &grp : by_dtype) {
        if (sbk_matvec_batch(grp.first, grp.second.data(), grp.second.size(), 0, c->stream))
            return fail("sbk_matvec_batch launch failed");
        c->stats.launches++;
    }
    if ((e = cudaMemcpyAsync(hs + xend, base + xend, yb, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(out)", e);
    if ((e = cudaStreamSynchronize(c->stream)) != cudaSuccess) return fail("cudaStreamSynchronize", e);
    cp.clear();
    for (size_t i = 0; i < nops; i++)
        if (res[i]) cp.push_back(HostCopy{ops[i].out, hs + yo[i], ops[i].rows * 4});
    c->copy(cp);
    for (size_t i = 0; i < nops; i++) done[i] = res[i] ? 1 : 0;
    c->stats.total_ns += now_ns() - t0;
    return 1;
}

extern "C" int sb_rmsnorm(sb_ctx *c, float *x, const float *w, size_t n, float eps)
{
    if (!c) return fail("null context");
    if (!x || !w) return fail("null argument");
    if (n == 0) return 0;
    std::lock_guard<std::mutex> lk(c->mu);
    cudaError_t e = cudaSetDevice(c->device);
    if (e != cudaSuccess) return fail("cudaSetDevice", e);
    const size_t b = (n * 4 + 255) & ~(size_t)255;
    if (c->ensure_scratch(2 * b) || c->ensure_host_stage(2 * b)) return -1;
    float *dx = (float *)c->scratch, *dw = (float *)((char *)c->scratch + b);
    char *hs = (char *)c->host_stage;
    memcpy(hs, x, n * 4);
    memcpy(hs + b, w, n * 4);
    if ((e = cudaMemcpyAsync(dx, hs, 2 * b, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync", e);
    if (sbk_rmsnorm(dx, nullptr, nullptr, dw, dx, 1, n, eps, c->stream)) return fail("sbk_rmsnorm launch failed");
    if ((e = cudaMemcpyAsync(hs, dx, n * 4, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync", e);
    if ((e = cudaStreamSynchronize(c->stream)) != cudaSuccess) return fail("cudaStreamSynchronize", e);
    memcpy(x, hs, n * 4);
    c->stats.launches++;
    return 1;
}
