// engine.cuh -- whole-token decode on the device: the model resident in HBM,
// one CUDA graph per token, positions and tokens read from device memory.
//
// The boundary is GpuDispatch::decode_preparar / decode_token
// (crates/soso-llm-core/src/gpu.rs:654-684) with the plan of gpu.rs:92-158.
// One token runs the reference's dense GQA layer (layer.rs:947-1398):
//   xn = rmsnorm(h, attn_norm)                         gemm.rs:93-100
//   q|k|v = W{q,k,v} . xn  (+ bias, QK-norm, RoPE)      layer.rs:1100-1193
//   append f16 K/V at pos; o = attention(q, K, V)      kv.rs:258-275, attn.rs:73-140
//   h += Wo . o ; xn = rmsnorm(h, ffn_norm)            layer.rs:1283-1311
//   h += Wdown . (silu(Wgate . xn) * (Wup . xn))        layer.rs:1352-1389
// then logits = lm_head . rmsnorm(h, final_norm) and, for greedy decoding,
// token = argmax(logits) (runtime.rs:1976-2028).  The residual add of each
// block is fused into the RMSNorm that follows it.
//
// Per token: 5 launches per layer + 2, all captured once.  Independent matvecs
// of one input (q/k/v, gate/up) share one launch (sbk_matvec_batch_x), and the
// elementwise steps are folded into the launches around them: the residual add
// and RMSNorm into the preparation of the next matvec's input, SwiGLU into the
// down projection's, bias / QK-norm / RoPE / KV append into attention, and the
// end of a greedy step into argmax.  The residual stream alternates between two
// buffers (a matvec's CTAs read one while CTA 0 writes the other).
#pragma once
#include <algorithm>
#include <vector>

#include "dispatch.cuh"
#include "decode_ops.cuh"

extern "C" int sbk_embed_row(const void *table, uint8_t dtype, size_t vocab, size_t hidden, const int32_t *token,
                             float *out, int pdl, void *stream);
extern "C" int sbk_rope_kv_append(float *qkv, const float *bias, const float *qnorm, const float *knorm,
                                  uint16_t *kcache, uint16_t *vcache, const int32_t *pos, size_t heads,
                                  size_t kv_heads, size_t head_dim, size_t ctx, float theta, float eps, int neox,
                                  int pdl, void *stream);
extern "C" size_t sbk_attn_ws_bytes(size_t heads, size_t kv_heads, size_t head_dim, size_t ctx);
extern "C" int sbk_attn_decode(const float *q, const uint16_t *kcache, const uint16_t *vcache, float *out,
                               const int32_t *pos, size_t heads, size_t kv_heads, size_t head_dim, size_t ctx,
                               void *ws, int pdl, void *stream);
extern "C" size_t sbk_argmax_ws_bytes(void);
extern "C" int sbk_argmax(const float *v, size_t n, int32_t *out, void *ws, int pdl, void *stream);
extern "C" int sbk_attn_rope_decode_yarn(const float *qkv, const float *bias, const float *qnorm, const float *knorm,
                                         uint16_t *kcache, uint16_t *vcache, float *out, const int32_t *pos,
                                         size_t heads, size_t kv_heads, size_t head_dim, size_t ctx, float theta,
                                         float eps, int neox, const float *factors, float mscale, void *ws, int pdl,
                                         void *stream);

namespace sb {

// silu(g) * u  (gemm.rs:210-226)
__global__ void swiglu_kernel(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ o, int n)
{
    griddep_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float x = g[i];
        o[i] = x / (1.0f + expf(-x)) * u[i];
    }
    griddep_launch();
}

// This token's cache rows of every layer into one contiguous buffer, in layer order:
// [k | v] for an attention layer, the latent row for an MLA layer.  One CTA per segment.
struct KvSeg {
    const uint16_t *src;  // cache [ctx][width]
    long long dst_off;
    int width, pad;
};

__global__ void kv_rows_kernel(const KvSeg *segs, const int *pos, uint16_t *out)
{
    griddep_wait();
    const KvSeg g = segs[blockIdx.x];
    const long long p = *pos;
    for (int i = threadIdx.x; i < g.width; i += blockDim.x) out[g.dst_off + i] = g.src[p * g.width + i];
}

// MoE routing of one token on the device, between the router matvec and the expert
// matvecs: softmax over all experts, stable top-k by weight, renormalised
// (gemm::topk_softmax, crates/soso-llm-core/src/gemm.rs:62-91, as router_topk_kernel),
// the shared expert's weight sigmoid(gate_row . x) or 1 (layer.rs:1883-1907), and the
// expert choice written into the device-side batches of the two expert launches.
// The choices whose experts are resident here (all of them on one GPU; the rank's range
// of expert IDs under expert parallelism) are taken in choice order; with m of them the
// launches run batch m of their k + 1 prepared batches, whose first m matrices (pairs for
// gate|up) now point at those experts' tensor maps and, for the downs, publish to the
// exchange slot of their choice.  One CTA.
struct RouteArgs {
    const float *logits;
    int n_exp, k;
    int *idx;
    float *wts;             // [k] routed weights, then the shared expert's weight
    const float *sg_row;    // shared expert gate row [H], or null (weight 1)
    const float *h;         // residual stream after attention (x = rmsnorm(h) * nw)
    const float *nw;
    float eps;
    int H, has_shared;
    tcmv::Batch *gu, *dn;   // [k + 1] each: batch m runs m resident choices (+ the shared
                            // expert, when it is computed here, as matrix m)
    int *sel;               // the batch index m, for both launches
    const CUtensorMap *maps;  // [hi - lo][3]: gate, up, down of the resident experts (pairs: gate/up, -, down)
    int lo, hi;             // resident experts [lo, hi)
    int pairs;              // gate|up launches run one gate/up pair matrix per choice
    int xw;                 // floats between exchange slots: the down of choice r publishes at r * xw
    // route trace of this layer: row *pos of RT_W ints (the chosen IDs in rank order, then at
    // RT_GAP the router-logit gap between the k-th and (k+1)-th choice, as float bits), rows
    // trace_row ints apart; read by sb_decode_routes / sb_decode_route_trace
    int *trace;
    const int *pos;
    int trace_row;
};
constexpr int RT_W = 17, RT_GAP = 16;

// The router of a MoE layer whose matrix is f32, as the reference stores ffn_gate_inp (its
// router matvec, layer.rs:1959-1972, runs in f32), with the input formed as the fused matvec
// forms it (XS_NORM): h = a + (res, or the weighted set of the previous MoE layer's outputs)
// -> h_out (CTA 0), x = rmsnorm(h) * w (gemm.rs:93-100); logits[e] = W[e] . x.  Every CTA
// forms x in shared memory itself and takes 8 experts, one per warp.
struct RouterF32Args {
    const float *a, *res, *ys, *yw;
    int ny, ystride;
    float *h_out;
    const float *nw;
    float eps;
    const float *W;
    float *logits;
    int H, n_exp;
};

__global__ void __launch_bounds__(256) router_f32_kernel(RouterF32Args r)
{
    extern __shared__ float xs[];  // [H]
    __shared__ float red[8];
    griddep_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < r.H; i += blockDim.x) {
        float v = r.a[i];
        if (r.ny) {
            float acc = 0.0f;
            for (int k = 0; k < r.ny; k++) acc += __ldcg(r.ys + (size_t)k * r.ystride + i) * r.yw[k];
            v = acc + v;
        } else if (r.res) {
            v += r.res[i];
        }
        xs[i] = v;
        ss += v * v;
        if (blockIdx.x == 0 && r.h_out) r.h_out[i] = v;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int w = 0; w < 8; w++) tot += red[w];
    const float scale = 1.0f / sqrtf(tot / (float)r.H + r.eps);
    for (int i = threadIdx.x; i < r.H; i += blockDim.x) xs[i] = xs[i] * scale * r.nw[i];
    __syncthreads();
    const int e = blockIdx.x * 8 + warp;
    if (e < r.n_exp) {
        const float *wr = r.W + (size_t)e * r.H;
        float acc = 0.0f;
        for (int i = lane; i < r.H; i += 32) acc += wr[i] * xs[i];
        acc = warp_sum(acc);
        if (lane == 0) r.logits[e] = acc;
    }
    griddep_launch();
}

__global__ void __launch_bounds__(256) route_kernel(RouteArgs a)
{
    __shared__ float p[1024];
    __shared__ float red[32];
    __shared__ float topw[64];
    __shared__ int topi[64];
    __shared__ int own[64];
    __shared__ int s_m, s_next;
    griddep_launch();  // the expert launches read the batches only after their own wait
    griddep_wait();
    const int tid = threadIdx.x, n = a.n_exp;
    float m = -INFINITY;
    for (int i = tid; i < n; i += blockDim.x) m = fmaxf(m, a.logits[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tid & 31) == 0) red[tid >> 5] = m;
    __syncthreads();
    m = -INFINITY;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) m = fmaxf(m, red[w]);
    __syncthreads();
    float sum = 0.0f;
    for (int i = tid; i < n; i += blockDim.x) {
        p[i] = expf(a.logits[i] - m);
        sum += p[i];
    }
    sum = warp_sum(sum);
    if ((tid & 31) == 0) red[tid >> 5] = sum;
    __syncthreads();
    sum = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); w++) sum += red[w];
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x)
        if (sum > 0.0f) p[i] = p[i] / sum;
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
        const float v = p[i];
        int r = 0;
        for (int j = 0; j < n; j++) {
            const float u = p[j];
            r += (u > v) || (u == v && j < i);
        }
        if (r < a.k) topi[r] = i, topw[r] = v;
        if (r == a.k) s_next = i;  // the best expert not chosen: its logit gap goes in the trace
    }
    // shared expert gate: sigmoid(row . rmsnorm(h) * nw), the dot in warp 0
    float sg = 1.0f;
    if (a.has_shared && a.sg_row) {
        float ss = 0.0f, dot = 0.0f;
        for (int i = tid; i < a.H; i += blockDim.x) ss += a.h[i] * a.h[i];
        ss = warp_sum(ss);
        __syncthreads();
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        __syncthreads();
        ss = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) ss += red[w];
        const float scale = 1.0f / sqrtf(ss / (float)a.H + a.eps);
        __syncthreads();
        for (int i = tid; i < a.H; i += blockDim.x) dot += a.sg_row[i] * (a.h[i] * scale * a.nw[i]);
        dot = warp_sum(dot);
        if ((tid & 31) == 0) red[tid >> 5] = dot;
        __syncthreads();
        dot = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) dot += red[w];
        sg = 1.0f / (1.0f + expf(-dot));
    }
    __syncthreads();
    if (tid == 0) {
        float t = 0.0f;
        for (int r = 0; r < a.k; r++) t += topw[r];
        int *tr = a.trace + (size_t)(*a.pos) * a.trace_row;
        for (int r = 0; r < a.k; r++) {
            a.wts[r] = t > 0.0f ? topw[r] / t : topw[r];
            a.idx[r] = topi[r];
            tr[r] = topi[r];
        }
        tr[RT_GAP] = __float_as_int(a.k < n ? a.logits[topi[a.k - 1]] - a.logits[s_next] : INFINITY);
        if (a.has_shared) a.wts[a.k] = sg;
        int mo = 0;
        for (int r = 0; r < a.k; r++)
            if (topi[r] >= a.lo && topi[r] < a.hi) own[mo++] = r;
        s_m = mo;
        *a.sel = mo;
    }
    __syncthreads();
    const int mo = s_m;  // resident choices: batch mo of the k + 1
    if (tid < mo) {
        const int r = own[tid], e = topi[r] - a.lo;
        tcmv::Batch *gu = a.gu + mo, *dn = a.dn + mo;
        if (a.pairs) {
            gu->d[tid].mapp = a.maps + 3 * e;
        } else {
            gu->d[2 * tid].mapp = a.maps + 3 * e;
            gu->d[2 * tid + 1].mapp = a.maps + 3 * e + 1;
        }
        dn->d[tid].mapp = a.maps + 3 * e + 2;
        dn->d[tid].pub_off = r * a.xw;
    }
}

}  // namespace sb

extern "C" int sbk_swiglu(const float *gate, const float *up, float *out, size_t n, int pdl, void *stream)
{
    if (!gate || !up || !out || n == 0 || n > (1u << 30)) return -1;
    const unsigned blocks = (unsigned)((n + 255) / 256 < 1184 ? (n + 255) / 256 : 1184);
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3(blocks);
    c.blockDim = dim3(256);
    c.stream = (cudaStream_t)stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    c.attrs = at;
    c.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&c, sb::swiglu_kernel, gate, up, out, (int)n) == cudaSuccess ? 0 : -4;
}

namespace {

struct EngMat {
    const void *w = nullptr;
    uint8_t dt = 0;
    size_t rows = 0, cols = 0;
};

struct EngLayer {
    EngMat q, k, v, o, g, u, d;
    EngMat gu2;  // gate and up as one matrix of 16-row group pairs (its launch forms silu(gate) * up)
    size_t heads = 0, kvh = 0, hd = 0, qd = 0, kvd = 0, ffn = 0;
    float theta = 0.0f;
    int neox = 0;
    float *qn = nullptr, *kn = nullptr, *bias = nullptr, *na = nullptr, *nf = nullptr;
    float *rf = nullptr;  // YaRN divisors [hd / 2] or null
    float rms = 1.0f;     // YaRN mscale
    uint16_t *kc = nullptr, *vc = nullptr;
    // MoE FFN (sb_moe_plan): router, n_exp experts (gate, up, down), optional shared expert
    bool moe = false, has_sh = false;
    size_t n_exp = 0, top_k = 0, effn = 0, sffn = 0;
    EngMat router, sh[3];
    std::vector<EngMat> ex;            // [hi - lo][3]: the resident experts
    size_t ex_lo = 0, ex_hi = 0;       // resident experts (all, or this rank's IDs)
    bool ex_pairs = false;             // ex[3x] (and sh[0]) is the gate/up pair matrix, ex[3x + 1] unused
    bool sh_here = false;              // the shared expert is computed on this GPU
    float *sg = nullptr;               // shared expert gate row, or null (weight 1)
    CUtensorMap *maps = nullptr;       // device [hi - lo][3]: the resident experts' tensor maps
    sb::tcmv::Batch *gu_b = nullptr;   // device batches of the two expert launches, [top_k + 1]
    sb::tcmv::Batch *dn_b = nullptr;   //   each (built on the first enqueue; the route kernel
    int *sel = nullptr;                //   picks one and its maps, and writes its index here)
    size_t gu_smem = 0, dn_smem = 0;
    const float *built_for = nullptr;  // residual buffer the batches read
    // tensor parallelism: attention heads / FFN blocks sharded (else computed whole here)
    bool tp_attn = false, tp_ffn = false;
    // MLA attention (sb_mla_plan): latent cache + rope keys instead of K/V rows
    bool mla = false;
    size_t q_rank = 0, kv_rank = 0, qk_nope = 0, qk_rope = 0, v_dim = 0;
    EngMat q_down, q_up, kv_down, k_up, v_up;
    uint16_t *latent = nullptr;
    float *krope = nullptr;
};

}  // namespace

struct sb_engine {
    std::vector<EngLayer> L;
    size_t H = 0, V = 0, ctx = 0, ffn_max = 0, qkv_max = 0, kv_rows_total = 0;
    float eps = 0.0f;
    EngMat lm, emb;
    float *fnorm = nullptr;
    float *hfin = nullptr;  // which residual buffer holds the hidden vector a step leaves (before the output norm)
    float *h = nullptr, *h2 = nullptr, *tmp = nullptr, *qkv = nullptr, *att = nullptr, *ob = nullptr, *gu = nullptr,
          *logits = nullptr;
    // MoE: router logits, chosen experts and weights, gate|up per choice, down outputs per choice
    float *rlog = nullptr, *wts = nullptr, *egu = nullptr, *ys = nullptr;
    int *ridx = nullptr;
    int *rtrace = nullptr;  // [ctx][layers][RT_W]: per decode position, the experts each MoE layer chose
    size_t last_pos = 0;    // position of the last decode step (host)
    bool traced = false;    // a decode step ran since prepare
    void *pf = nullptr;     // block prefill state (prefill_engine.cuh)
    size_t moe_slots = 0, moe_ffn = 0, n_exp_max = 0;
    // MLA: q_down | kv_down outputs, q_up output, absorbed query, roped q slice, latent sums
    float *mcq = nullptr, *mc = nullptr, *mq = nullptr, *mqt = nullptr, *mqr = nullptr, *mcbar = nullptr;
    size_t mla_q = 0, mla_r = 0, mla_qq = 0, mla_hr = 0, mla_hp = 0;
    void *mla_ws = nullptr;
    size_t mla_ws_bytes = 0;
    void *kv_segs = nullptr;
    size_t n_kv_segs = 0;
    // tensor parallelism (sb_group of world > 1): this rank's vocabulary slice of the output
    sb_group *tp = nullptr;
    size_t vbase = 0, vn = 0;
    size_t attn_ws_bytes = 0;
    bool pending_finish = false;  // sb_decode_finish still to run (warm-up + capture)
    int *ints = nullptr;  // pos, tok, step, n_prompt
    int *prompt = nullptr, *hist = nullptr;
    void *attn_ws = nullptr, *am_ws = nullptr;
    uint16_t *kv_rows = nullptr;
    std::vector<void *> allocs;
    cudaGraphExec_t g_tok = nullptr, g_greedy = nullptr;
    size_t launches_per_token = 0;

    void *dalloc(size_t bytes, cudaError_t *e)
    {
        void *p = nullptr;
        *e = cudaMalloc(&p, bytes ? bytes : 16);
        if (*e == cudaSuccess) allocs.push_back(p);
        return p;
    }
    ~sb_engine()
    {
        if (pf) sb_pf_free(pf);
        if (g_tok) cudaGraphExecDestroy(g_tok);
        if (g_greedy) cudaGraphExecDestroy(g_greedy);
        for (void *p : allocs) cudaFree(p);
    }
};

void sb_engine_free(sb_engine *e) { delete e; }

namespace {

// Resident weight of a plan matrix (uploaded on first sight under its key).
int eng_mat(sb_ctx *c, const sb_mat &m, size_t rows, size_t cols, EngMat *out, bool matvec)
{
    if (!m.key || !m.view.bytes) return fail("decode plan: matrix without key or bytes");
    if (m.rows != rows || m.cols != cols) return fail(std::string("decode plan: ") + m.key + " has an unexpected shape");
    if (matvec && !admit(&m.view, rows, cols)) return 0;
    Resident *r = nullptr;
    const int rc = c->resident(m.key, &m.view, rows, cols, &r, matvec);
    if (rc <= 0) return rc;
    out->w = r->ptr;
    out->dt = r->dev_dtype;
    out->rows = rows;
    out->cols = cols;
    return 1;
}

// Rows [r0, r0 + nr) of a plan matrix (a tensor-parallel shard), resident under its own key.
int eng_mat_rows(sb_ctx *c, const sb_mat &m, size_t rows, size_t cols, size_t r0, size_t nr, EngMat *out)
{
    if (!m.key || !m.view.bytes) return fail("decode plan: matrix without key or bytes");
    if (m.rows != rows || m.cols != cols) return fail(std::string("decode plan: ") + m.key + " has an unexpected shape");
    if (!admit(&m.view, rows, cols) || r0 + nr > rows || !nr) return 0;
    const size_t rb = sbk_row_bytes(m.view.dtype, cols);
    sb_view v = m.view;
    v.bytes += r0 * rb;
    v.len = nr * rb;
    v.elems = nr * cols;
    const std::string key = std::string(m.key) + "#rows" + std::to_string(r0) + "+" + std::to_string(nr);
    Resident *r = nullptr;
    const int rc = c->resident(key.c_str(), &v, nr, cols, &r, true);
    if (rc <= 0) return rc;
    *out = EngMat{r->ptr, r->dev_dtype, nr, cols};
    return 1;
}

// Columns [c0, c0 + nc) of a plan matrix (whole blocks: a tensor-parallel shard of its input
// dimension), gathered row by row on the host, resident under its own key.
int eng_mat_cols(sb_ctx *c, const sb_mat &m, size_t rows, size_t cols, size_t c0, size_t nc, EngMat *out)
{
    if (!m.key || !m.view.bytes) return fail("decode plan: matrix without key or bytes");
    if (m.rows != rows || m.cols != cols) return fail(std::string("decode plan: ") + m.key + " has an unexpected shape");
    if (!admit(&m.view, rows, cols) || c0 + nc > cols || !nc) return 0;
    const uint8_t dt = m.view.dtype;
    const size_t rb = sbk_row_bytes(dt, cols), ob = c0 ? sbk_row_bytes(dt, c0) : 0, sb_ = sbk_row_bytes(dt, nc);
    if (!sb_ || (c0 && !ob)) return 0;  // not on block boundaries
    std::vector<uint8_t> tmp(rows * sb_);
    for (size_t r = 0; r < rows; r++) memcpy(tmp.data() + r * sb_, m.view.bytes + r * rb + ob, sb_);
    sb_view v{tmp.data(), tmp.size(), dt, rows * nc};
    const std::string key = std::string(m.key) + "#cols" + std::to_string(c0) + "+" + std::to_string(nc);
    Resident *r = nullptr;
    const int rc = c->resident(key.c_str(), &v, rows, nc, &r, true);
    if (rc <= 0) return rc;
    *out = EngMat{r->ptr, r->dev_dtype, rows, nc};
    return 1;
}

// Rows [r0, r0 + nr) of a gate and an up matrix as one matrix of 16-row groups of each in
// turn (gate rows 16p.., then up rows 16p.., for p = 0, 1, ...): the launch over it forms
// silu(gate) * up in its epilogue.  Resident under its own key; 0 when the pair does not
// qualify (different dtypes, rows not whole groups, a format without the tensor-core kernel).
int eng_mat_pairs(sb_ctx *c, const sb_mat &g, const sb_mat &u, size_t rows, size_t cols, size_t r0, size_t nr,
                  EngMat *out)
{
    if (!g.key || !u.key || !g.view.bytes || !u.view.bytes) return fail("decode plan: matrix without key or bytes");
    if (g.rows != rows || g.cols != cols || u.rows != rows || u.cols != cols)
        return fail(std::string("decode plan: ") + g.key + " / " + u.key + " have unexpected shapes");
    const uint8_t dt = g.view.dtype;
    if (dt != u.view.dtype || nr % 16 || !nr || r0 + nr > rows || !admit(&g.view, rows, cols) ||
        !admit(&u.view, rows, cols))
        return 0;
    if (dt != SB_DTYPE_Q4_K && dt != SB_DTYPE_Q6_K && dt != SB_DTYPE_Q8_0) return 0;
    const size_t rb = sbk_row_bytes(dt, cols);
    if (!rb) return 0;
    std::vector<uint8_t> tmp(2 * nr * rb);
    for (size_t p = 0; p < nr / 16; p++) {
        memcpy(tmp.data() + (2 * p) * 16 * rb, g.view.bytes + (r0 + 16 * p) * rb, 16 * rb);
        memcpy(tmp.data() + (2 * p + 1) * 16 * rb, u.view.bytes + (r0 + 16 * p) * rb, 16 * rb);
    }
    sb_view v{tmp.data(), tmp.size(), dt, 2 * nr * cols};
    const std::string key = std::string(g.key) + "|" + u.key + "#pairs" + std::to_string(r0) + "+" + std::to_string(nr);
    Resident *r = nullptr;
    const int rc = c->resident(key.c_str(), &v, 2 * nr, cols, &r, true);
    if (rc <= 0) return rc;
    if (r->dev_dtype != SB_DTYPE_Q4_K && r->dev_dtype != SB_DTYPE_Q6_K_P && r->dev_dtype != SB_DTYPE_Q8_0_R) return 0;
    *out = EngMat{r->ptr, r->dev_dtype, 2 * nr, cols};
    return 1;
}

int upload_f32(sb_engine *e, const float *src, size_t n, float **dst)
{
    *dst = nullptr;
    if (!src) return 0;
    cudaError_t err;
    float *p = (float *)e->dalloc(n * 4, &err);
    if (err != cudaSuccess) return fail("cudaMalloc(plan vector)", err);
    if ((err = cudaMemcpy(p, src, n * 4, cudaMemcpyHostToDevice)) != cudaSuccess) return fail("cudaMemcpy(plan)", err);
    *dst = p;
    return 0;
}

bool fused_dtype(uint8_t dt)
{
    return dt == SB_DTYPE_Q4_K || dt == SB_DTYPE_Q6_K_P || dt == SB_DTYPE_Q8_0 || dt == SB_DTYPE_Q8_0_R;
}

// The matvecs `ms` (one input vector a, outputs ys) with the input formed as xs says:
// one fused launch per dtype where the kernel has the fused input forms, else the
// input is materialised first (sbk_rmsnorm / sbk_swiglu into `tmp`).
int run_mv(sb_engine *e, const EngMat *const *ms, float *const *ys, int n, const float *a, const sbk_xsrc &xs,
           cudaStream_t s, size_t *launches, const sb::grp::Pub *pub = nullptr, const sb::grp::Wait *wait = nullptr,
           bool pairs = false)
{
    if ((pub && pub->n) || (wait && wait->n) || pairs) {
        // tensor-parallel forms: one dtype, the tensor-core kernels only
        sbk_mv_op ops[8];
        for (int j = 0; j < n; j++) {
            if (ms[j]->dt != ms[0]->dt) return -5;
            ops[j] = sbk_mv_op{ms[j]->w, ms[j]->rows, ms[j]->cols, a, ys[j]};
        }
        const sb::tcmv::XSrc x{xs.res, xs.norm_w, xs.h_out, xs.eps, xs.mode, xs.ys, xs.yw, xs.ny, xs.ystride};
        const int rc = sb::matvec_batch_group(ms[0]->dt, ops, n, x, pub, wait, s, pairs);
        if (rc) return rc;
        *launches += 1;
        return 0;
    }
    bool done[8] = {false};
    for (int i = 0; i < n; i++) {
        if (done[i]) continue;
        const uint8_t dt = ms[i]->dt;
        sbk_mv_op ops[8];
        int k = 0;
        for (int j = i; j < n; j++)
            if (!done[j] && ms[j]->dt == dt) ops[k++] = sbk_mv_op{ms[j]->w, ms[j]->rows, ms[j]->cols, a, ys[j]}, done[j] = true;
        int rc;
        if (fused_dtype(dt) || xs.mode == SBK_XS_PLAIN) {
            rc = xs.mode == SBK_XS_PLAIN ? sbk_matvec_batch(dt, ops, k, 1, s) : sbk_matvec_batch_x(dt, ops, k, &xs, 1, s);
        } else {
            const size_t cols = ops[0].cols;
            if (xs.ny) return -5;  // the weighted residual set exists only in the fused form
            if (xs.mode == SBK_XS_NORM)
                rc = sbk_rmsnorm(a, xs.res, xs.res ? xs.h_out : nullptr, xs.norm_w, e->tmp, 1, cols, xs.eps, s);
            else
                rc = sbk_swiglu(a, xs.res, e->tmp, cols, 1, s);
            if (rc) return rc;
            *launches += 1;
            for (int j = 0; j < k; j++) ops[j].x = e->tmp;
            rc = sbk_matvec_batch(dt, ops, k, 1, s);
        }
        if (rc) return rc;
        *launches += 1;
    }
    return 0;
}

// Build (once, eagerly, outside any capture) the device-side batches of a MoE layer's two
// expert launches, one pair per count m of routed choices resident here (only m = top_k on
// one GPU): gate|up of each (input rmsnorm(hc) * ffn_norm) and their downs (input
// silu(gate) * up per choice), with the shared expert last when it is computed here.
// Matrices of routed choices start out pointing at the first resident expert; route_kernel
// points them at the chosen ones.  Under expert parallelism (pub set) every down batch
// publishes its rows to the exchange slot of its choice (the shared expert's: slot top_k).
template <class FG, class FD>
int build_moe_batches(sb_engine *e, EngLayer &L, const float *hc, const sb::grp::Pub *pub)
{
    using namespace sb::tcmv;
    const int grid = sb::num_sms_cached();
    const int k = (int)L.top_k, sh = L.sh_here ? 1 : 0;
    const int m0 = pub ? 0 : k;
    XSrc xg{};
    xg.w = L.nf, xg.eps = e->eps, xg.mode = XS_NORM;
    XSrc xd{};
    xd.mode = L.ex_pairs ? XS_PLAIN : XS_SWIGLU;
    std::vector<Batch> hg(k + 1), hd(k + 1);
    memset(hg.data(), 0, hg.size() * sizeof(Batch));
    memset(hd.data(), 0, hd.size() * sizeof(Batch));
    size_t gs = 0, ds = 0;
    for (int m = m0; m <= k; m++) {
        const int ns = m + sh;
        size_t sg = 0, sd = 0;
        if (!ns) {
            empty_batch<FG>(&hg[m], xg, &sg);
            empty_batch<FD>(&hd[m], xd, &sd);
        } else {
            MatOpX gu[MAXB], dn[MAXB];
            for (int i = 0; i < ns; i++) {
                const bool shared = i == m;
                const EngMat &g = shared ? L.sh[0] : L.ex[0], &u = shared ? L.sh[1] : L.ex[1];
                const EngMat &d = shared ? L.sh[2] : L.ex[2];
                float *gi = e->egu + (size_t)(2 * i) * e->moe_ffn, *ui = e->egu + (size_t)(2 * i + 1) * e->moe_ffn;
                float *yi = e->ys + (size_t)(shared ? k : i) * e->H;
                if (L.ex_pairs) {  // one pair matrix per choice; its output is silu(gate) * up
                    gu[i] = MatOpX{MatOp{g.w, (int)g.rows, (int)g.cols, hc, gi}, nullptr, nullptr, 1};
                    dn[i] = MatOpX{MatOp{d.w, (int)d.rows, (int)d.cols, gi, yi}, nullptr, nullptr};
                    continue;
                }
                gu[2 * i] = MatOpX{MatOp{g.w, (int)g.rows, (int)g.cols, hc, gi}, nullptr, nullptr};
                gu[2 * i + 1] = MatOpX{MatOp{u.w, (int)u.rows, (int)u.cols, hc, ui}, nullptr, nullptr};
                dn[i] = MatOpX{MatOp{d.w, (int)d.rows, (int)d.cols, gi, yi}, ui, nullptr};
            }
            int rc = build_batch<FG>(gu, L.ex_pairs ? ns : 2 * ns, CNT_MAX, grid, &xg, &hg[m], &sg);
            if (rc) return fail("decode plan: expert gate/up batch rejected (" + std::to_string(rc) + ")");
            rc = build_batch<FD>(dn, ns, CNT_MAX, grid, &xd, &hd[m], &sd);
            if (!rc && pub) rc = whole_groups<FD>(&hd[m], grid, &sd);
            if (rc) return fail("decode plan: expert down batch rejected (" + std::to_string(rc) + ")");
            if (sh) hd[m].d[m].pub_off = k * sb::grp::XW;
        }
        if (pub) hd[m].pub = *pub;
        gs = std::max(gs, sg);
        ds = std::max(ds, sd);
    }
    cudaError_t err;
    if (!L.gu_b) {
        L.gu_b = (Batch *)e->dalloc((k + 1) * sizeof(Batch), &err);
        if (err == cudaSuccess) L.dn_b = (Batch *)e->dalloc((k + 1) * sizeof(Batch), &err);
        if (err == cudaSuccess) L.sel = (int *)e->dalloc(16, &err);
        if (err != cudaSuccess) return fail("cudaMalloc(batch)", err);
    }
    if ((err = cudaMemcpy(L.gu_b, hg.data(), (k + 1) * sizeof(Batch), cudaMemcpyHostToDevice)) != cudaSuccess ||
        (err = cudaMemcpy(L.dn_b, hd.data(), (k + 1) * sizeof(Batch), cudaMemcpyHostToDevice)) != cudaSuccess)
        return fail("cudaMemcpy(batch)", err);
    L.gu_smem = gs, L.dn_smem = ds;
    L.built_for = hc;
    return 0;
}

template <class F>
int launch_moe_batch(sb::tcmv::Batch *b, const int *sel, size_t smem, cudaStream_t s)
{
    using namespace sb::tcmv;
    const int grid = sb::num_sms_cached();
    void *ws = sb::stream_ws(s, ws_bytes(grid));
    if (!ws) return -3;
    return launch_dev_batch<F>(b, sel, smem, ws_of(ws), grid, 1, s);
}

// The MoE FFN after its router matvec: route, expert gate|up, expert downs.  pub: where the
// downs publish (expert parallelism), else null.
int moe_dispatch(sb_engine *e, EngLayer &L, const float *hc, cudaStream_t s, bool build, size_t *n,
                 const sb::grp::Pub *pub)
{
    const uint8_t gdt = L.ex[0].dt, ddt = L.ex[2].dt;
    int rc = 0;
    if (build) {
        const bool d80 = ddt == SB_DTYPE_Q8_0 || ddt == SB_DTYPE_Q8_0_R;
        using namespace sb::tcmv;
        if (gdt == SB_DTYPE_Q4_K && d80) rc = build_moe_batches<Q4K, Q80>(e, L, hc, pub);
        else if (gdt == SB_DTYPE_Q6_K_P && d80) rc = build_moe_batches<Q6KP, Q80>(e, L, hc, pub);
        else if (gdt == SB_DTYPE_Q4_K && ddt == SB_DTYPE_Q4_K) rc = build_moe_batches<Q4K, Q4K>(e, L, hc, pub);
        else if (gdt == SB_DTYPE_Q4_K && ddt == SB_DTYPE_Q6_K_P) rc = build_moe_batches<Q4K, Q6KP>(e, L, hc, pub);
        else if (gdt == SB_DTYPE_Q6_K_P && ddt == SB_DTYPE_Q6_K_P) rc = build_moe_batches<Q6KP, Q6KP>(e, L, hc, pub);
        else if (gdt == SB_DTYPE_Q6_K_P && ddt == SB_DTYPE_Q4_K) rc = build_moe_batches<Q6KP, Q4K>(e, L, hc, pub);
        else return fail("decode plan: expert dtypes without a tensor-core kernel");
        if (rc) return rc;
    }
    sb::RouteArgs ra{e->rlog, (int)L.n_exp, (int)L.top_k, e->ridx, e->wts, L.sg, hc, L.nf, e->eps, (int)e->H,
                     L.has_sh ? 1 : 0, L.gu_b, L.dn_b, L.sel, L.maps, (int)L.ex_lo, (int)L.ex_hi, L.ex_pairs ? 1 : 0,
                     sb::grp::XW, e->rtrace + (&L - e->L.data()) * sb::RT_W, e->ints,
                     (int)(e->L.size() * sb::RT_W)};
    if ((rc = sb::launch_k(sb::route_kernel, dim3(1), dim3(256), 0, 1, s, ra))) return rc;
    *n += 1;
    rc = gdt == SB_DTYPE_Q4_K ? launch_moe_batch<sb::tcmv::Q4K>(L.gu_b, L.sel, L.gu_smem, s)
                              : launch_moe_batch<sb::tcmv::Q6KP>(L.gu_b, L.sel, L.gu_smem, s);
    if (rc) return rc;
    *n += 1;
    rc = ddt == SB_DTYPE_Q4_K   ? launch_moe_batch<sb::tcmv::Q4K>(L.dn_b, L.sel, L.dn_smem, s)
         : ddt == SB_DTYPE_Q6_K_P ? launch_moe_batch<sb::tcmv::Q6KP>(L.dn_b, L.sel, L.dn_smem, s)
                                  : launch_moe_batch<sb::tcmv::Q80>(L.dn_b, L.sel, L.dn_smem, s);
    if (rc) return rc;
    *n += 1;
    return 0;
}

#define ENG_CHECK(x)                                                                                         \
    do {                                                                                                     \
        const int _rc = (x);                                                                                 \
        if (_rc) return fail(std::string("decode step: ") + #x + " rejected (" + std::to_string(_rc) + ")"); \
        n++;                                                                                                 \
    } while (0)
#define ENG_MV(...)                                                                                          \
    do {                                                                                                     \
        const int _rc = run_mv(e, __VA_ARGS__, s, &n);                                                        \
        if (_rc) return fail(std::string("decode step: matvec launch rejected (") + std::to_string(_rc) + ")"); \
    } while (0)
#define ENG_MV_G(PUB, WAIT, ...)                                                                             \
    do {                                                                                                     \
        const int _rc = run_mv(e, __VA_ARGS__, s, &n, PUB, WAIT);                                             \
        if (_rc) return fail(std::string("decode step: matvec launch rejected (") + std::to_string(_rc) + ")"); \
    } while (0)

// One token, enqueued on s.  greedy: embedding row from the device token, and
// argmax (which also ends the step) at the end.
//
// The residual stream: h (hc) plus what the last block produced, added in the preparation
// of the next block's input (rmsnorm(h + y) * w).  y is the attention or dense FFN output
// (ob), or the weighted expert outputs (ys, wts) of a MoE FFN, or, on a group of GPUs, the
// slots of an exchange point: the ranks' partial sums (tensor parallelism, weights 1) or
// the routed experts' outputs by choice (expert parallelism, the routing weights).
int enqueue_token(sb_engine *e, cudaStream_t s, bool greedy)
{
    size_t n = 0;
    int *pos = e->ints, *tok = e->ints + 1, *step = e->ints + 2, *np = e->ints + 3;
    float *hc = e->h, *ho = e->h2;  // residual stream: current / the other buffer
    if (greedy) ENG_CHECK(sbk_embed_row(e->emb.w, e->emb.dt, e->V, e->H, tok, e->h, 1, s));
    int moe_ny = 0;  // > 0: the last FFN was MoE, computed here; its result is the weighted set ys / wts
    // Exchange points of this token are numbered in the order they are published: the data
    // slots alternate with that number's parity, which is safe because no rank publishes
    // point x + 2 before every rank has read point x (to publish x + 1, every rank has read x
    // first, and x + 2 comes after waiting for all of x + 1).
    sb_group *const g = e->tp;
    const int G = g ? g->world : 1, grid = sb::num_sms_cached();
    int nx = 0;                  // exchange points published so far
    int xprev = -1;              // the exchange point holding the pending residual (-1: none)
    const float *xw = nullptr;   // its slots' weights
    int xny = 0;                 // and count
    auto pub_slot = [&](int x, int slot) {
        sb::grp::Pub pb{};
        pb.n = G;
        for (int p = 0; p < G; p++)
            pb.dst[p] = sb::grp::data_slot(g->peer[p], x, slot), pb.cnt[p] = sb::grp::cnt_slot(g->peer[p], x, g->rank);
        return pb;
    };
    auto wait_of = [&](int x) {
        sb::grp::Wait w{};
        if (g && x >= 0) w = sb::grp::Wait{sb::grp::cnt_slot(g->area, x, 0), g->epoch, G, grid};
        return w;
    };
    auto norm_src = [&](const float *w, float *h_out) {
        sbk_xsrc xs{};
        xs.norm_w = w, xs.h_out = h_out, xs.eps = e->eps, xs.mode = SBK_XS_NORM;
        if (g && xprev >= 0)
            xs.ys = sb::grp::data_slot(g->area, xprev, 0), xs.yw = xw, xs.ny = xny, xs.ystride = sb::grp::XW;
        else if (moe_ny) xs.ys = e->ys, xs.yw = e->wts, xs.ny = moe_ny, xs.ystride = (int)e->H;
        else xs.res = e->ob;
        return xs;
    };
    // consume the pending residual (after the launch that read it)
    auto consumed = [&]() { moe_ny = 0, xprev = -1, xw = nullptr, xny = 0; };
    for (size_t l = 0; l < e->L.size(); l++) {
        EngLayer &L = e->L[l];
        if (L.mla) {
            // MLA block: h (+ previous FFN output) -> rmsnorm -> q_down | kv_down; q_up;
            // absorbed query + latent / rope-key append; attention over the latent cache;
            // per head W_v,h . cbar_h
            {
                sbk_xsrc xs = norm_src(L.na, l ? ho : nullptr);
                if (!l) xs.res = nullptr;
                const EngMat *ms[2] = {&L.q_down, &L.kv_down};
                float *ys[2] = {e->mcq, e->mc};
                const sb::grp::Wait w = wait_of(l ? xprev : -1);
                ENG_MV_G(nullptr, &w, ms, ys, 2, hc, xs);
                if (l) std::swap(hc, ho);
                consumed();
            }
            {
                const sbk_xsrc xs{};
                const EngMat *ms[1] = {&L.q_up};
                float *ys[1] = {e->mq};
                ENG_MV(ms, ys, 1, e->mcq, xs);
            }
            ENG_CHECK(sbk_mla_absorb(e->mq, e->mc, L.k_up.w, L.k_up.dt, L.latent, L.krope, e->mqt, e->mqr, pos,
                                     L.heads, L.kvh, L.kv_rank, L.qk_nope, L.qk_rope, e->ctx, L.theta, 1, s));
            ENG_CHECK(sbk_mla_attn(e->mqt, e->mqr, L.latent, L.krope, e->mcbar, pos, L.heads, L.kvh, L.kv_rank,
                                   L.qk_nope, L.qk_rope, e->ctx, e->mla_ws, 1, s));
            {
                const size_t rb = sbk_row_bytes(L.v_up.dt, L.kv_rank);
                sbk_mv_op ops[sb::mla::MAXH];
                for (size_t h = 0; h < L.heads; h++) {
                    const size_t kvh = h / (L.heads / L.kvh);
                    ops[h] = sbk_mv_op{(const uint8_t *)L.v_up.w + kvh * L.v_dim * rb, L.v_dim, L.kv_rank,
                                       e->mcbar + h * L.kv_rank, e->att + h * L.v_dim};
                }
                ENG_CHECK(sbk_matvec_batch(L.v_up.dt, ops, L.heads, 1, s));
            }
        } else {
            // attention block: h (+ previous FFN output) -> rmsnorm -> q|k|v
            {
                sbk_xsrc xs = norm_src(L.na, l ? ho : nullptr);
                if (!l) xs.res = nullptr;
                const EngMat *ms[3] = {&L.q, &L.k, &L.v};
                float *ys[3] = {e->qkv, e->qkv + L.qd, e->qkv + L.qd + L.kvd};
                const sb::grp::Wait w = wait_of(l ? xprev : -1);
                ENG_MV_G(nullptr, &w, ms, ys, 3, hc, xs);
                if (l) std::swap(hc, ho);
                consumed();
            }
            ENG_CHECK(sbk_attn_rope_decode_yarn(e->qkv, L.bias, L.qn, L.kn, L.kc, L.vc, e->att, pos, L.heads, L.kvh,
                                                L.hd, e->ctx, L.theta, e->eps, L.neox, L.rf, L.rms, e->attn_ws, 1, s));
        }
        {
            const sbk_xsrc xs{};
            const EngMat *ms[1] = {&L.o};
            float *ys[1] = {e->ob};
            if (L.tp_attn) {  // this rank's heads' share of attn_output: to every rank
                const sb::grp::Pub pb = pub_slot(nx, g->rank);
                ENG_MV_G(&pb, nullptr, ms, ys, 1, e->att, xs);
                xprev = nx++, xw = g->ones, xny = G;
            } else {
                ENG_MV(ms, ys, 1, e->att, xs);
            }
        }
        if (L.moe) {
            // MoE FFN: h + attention output -> rmsnorm -> router logits; route; experts
            if (L.router.dt == SB_DTYPE_F32) {  // (one GPU only: prepare declines it in a group)
                const sbk_xsrc xs = norm_src(L.nf, ho);
                sb::RouterF32Args ra{hc, xs.res, xs.ys, xs.yw, xs.ny, xs.ystride, ho, L.nf, e->eps,
                                     (const float *)L.router.w, e->rlog, (int)e->H, (int)L.n_exp};
                ENG_CHECK(sb::launch_k(sb::router_f32_kernel, dim3((unsigned)((L.n_exp + 7) / 8)), dim3(256),
                                       e->H * 4, 1, s, ra));
                std::swap(hc, ho);
                consumed();
            } else {
                const sbk_xsrc xs = norm_src(L.nf, ho);
                const EngMat *ms[1] = {&L.router};
                float *ys[1] = {e->rlog};
                const sb::grp::Wait w = wait_of(xprev);
                ENG_MV_G(nullptr, &w, ms, ys, 1, hc, xs);
                std::swap(hc, ho);
                consumed();
            }
            const bool build = L.built_for == nullptr;
            if (!build && L.built_for != hc) return fail("decode step: MoE batches built for another buffer");
            const int ny = (int)(L.top_k + (L.has_sh ? 1 : 0));
            if (g) {  // expert parallelism: every choice's output to its slot of every rank's area
                const sb::grp::Pub pb = pub_slot(nx, 0);
                if (moe_dispatch(e, L, hc, s, build, &n, &pb)) return fail("decode step: MoE launch rejected");
                xprev = nx++, xw = e->wts, xny = ny;
            } else {
                if (moe_dispatch(e, L, hc, s, build, &n, nullptr)) return fail("decode step: MoE launch rejected");
                moe_ny = ny;
            }
            continue;
        }
        // dense FFN block: h + attention output -> rmsnorm -> gate|up; silu(gate) * up -> down
        // (with the gate/up pairs matrix, its launch forms silu(gate) * up itself)
        if (L.gu2.w) {
            const sbk_xsrc xs = norm_src(L.nf, ho);
            const EngMat *ms[1] = {&L.gu2};
            float *ys[1] = {e->gu};
            const sb::grp::Wait w = wait_of(xprev);
            const int rc = run_mv(e, ms, ys, 1, hc, xs, s, &n, nullptr, &w, true);
            if (rc) return fail("decode step: gate/up launch rejected (" + std::to_string(rc) + ")");
            std::swap(hc, ho);
            consumed();
        } else {
            const sbk_xsrc xs = norm_src(L.nf, ho);
            const EngMat *ms[2] = {&L.g, &L.u};
            float *ys[2] = {e->gu, e->gu + L.ffn};
            const sb::grp::Wait w = wait_of(xprev);
            ENG_MV_G(nullptr, &w, ms, ys, 2, hc, xs);
            std::swap(hc, ho);
            consumed();
        }
        {
            sbk_xsrc xs{};
            if (!L.gu2.w) xs.res = e->gu + L.ffn, xs.mode = SBK_XS_SWIGLU;
            const EngMat *ms[1] = {&L.d};
            float *ys[1] = {e->ob};
            if (L.tp_ffn) {  // this rank's share of ffn_down: to every rank
                const sb::grp::Pub pb = pub_slot(nx, g->rank);
                ENG_MV_G(&pb, nullptr, ms, ys, 1, e->gu, xs);
                xprev = nx++, xw = g->ones, xny = G;
            } else {
                ENG_MV(ms, ys, 1, e->gu, xs);
            }
        }
    }
    {
        // the residual stream's last value goes to the other buffer on the way (the hidden
        // vector of the step, Runtime::hidden)
        const sbk_xsrc xs = norm_src(e->fnorm, ho);
        e->hfin = ho;
        const EngMat *ms[1] = {&e->lm};
        float *ys[1] = {e->logits};
        const sb::grp::Wait w = wait_of(xprev);
        ENG_MV_G(nullptr, &w, ms, ys, 1, hc, xs);
    }
    if (greedy && g) {
        // the maximum of this rank's vocabulary slice to every rank, then the global one
        const int xa = nx;
        sb::grp::Pub pb{};
        pb.n = G;
        for (int p = 0; p < G; p++)
            pb.dst[p] = reinterpret_cast<float *>(sb::grp::arg_slot(g->peer[p], g->rank)),
            pb.cnt[p] = sb::grp::cnt_slot(g->peer[p], xa, g->rank);
        unsigned *cnt = (unsigned *)e->am_ws;
        float *pv = (float *)((char *)e->am_ws + 256);
        int *pi = (int *)((char *)e->am_ws + 256 + sb::AM_GRID * 8);
        sb::ArgmaxArgs aa{e->logits, (int)e->vn, pv, pi, cnt, tok, nullptr, nullptr, nullptr, nullptr, nullptr,
                          (int)e->vbase, pb};
        ENG_CHECK(sb::launch_k(sb::argmax_kernel, dim3(sb::AM_GRID), dim3(sb::AM_THREADS), 0, 1, s, aa));
        sb::GatherArgs ga{g->area, sb::grp::cnt_slot(g->area, xa, 0), g->epoch, G, tok, pos, step, e->hist, e->prompt, np};
        ENG_CHECK(sb::launch_k(sb::argmax_gather_kernel, dim3(1), dim3(32), 0, 1, s, ga));
    } else if (greedy) {
        ENG_CHECK(sb::argmax_launch(e->logits, e->vn, tok, e->am_ws, 1, s, pos, step, e->hist, e->prompt, np));
    } else {
        sb::kv_rows_kernel<<<(unsigned)e->n_kv_segs, 256, 0, s>>>((const sb::KvSeg *)e->kv_segs, pos, e->kv_rows);
        if (cudaGetLastError() != cudaSuccess) return fail("decode step: kv rows launch failed");
        n++;
    }
    e->launches_per_token = n;
    return 0;
}

int capture(sb_engine *e, cudaStream_t s, bool greedy, cudaGraphExec_t *out)
{
    cudaGraph_t g = nullptr;
    cudaError_t err = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    if (err != cudaSuccess) return fail("cudaStreamBeginCapture", err);
    const int rc = enqueue_token(e, s, greedy);
    err = cudaStreamEndCapture(s, &g);
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (err != cudaSuccess) return fail("cudaStreamEndCapture", err);
    err = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (err != cudaSuccess) return fail("cudaGraphInstantiate", err);
    return 0;
}

// Positions, tokens, KV caches and the split-K workspaces back to zero (the group's epoch
// and exchange counters are never reset).
cudaError_t engine_zero(sb_engine *e, cudaStream_t s)
{
    cudaError_t z = cudaMemsetAsync(e->ints, 0, 64, s);
    for (auto &L : e->L) {
        if (L.mla) {
            if (z == cudaSuccess) z = cudaMemsetAsync(L.latent, 0, e->ctx * L.kv_rank * 2, s);
            if (z == cudaSuccess) z = cudaMemsetAsync(L.krope, 0, e->ctx * L.kvh * L.qk_rope * 4, s);
            continue;
        }
        if (z == cudaSuccess) z = cudaMemsetAsync(L.kc, 0, e->ctx * L.kvd * 2, s);
        if (z == cudaSuccess) z = cudaMemsetAsync(L.vc, 0, e->ctx * L.kvd * 2, s);
    }
    if (z == cudaSuccess && e->mla_ws) z = cudaMemsetAsync(e->mla_ws, 0, e->mla_ws_bytes, s);
    if (z == cudaSuccess && e->attn_ws_bytes) z = cudaMemsetAsync(e->attn_ws, 0, e->attn_ws_bytes, s);
    if (z == cudaSuccess) z = cudaMemsetAsync(e->am_ws, 0, sbk_argmax_ws_bytes(), s);
    if (z == cudaSuccess) z = cudaMemsetAsync(e->h, 0, e->H * 4, s);
    if (z == cudaSuccess) z = cudaStreamSynchronize(s);
    return z;
}

}  // namespace

extern "C" int sb_decode_prepare(sb_ctx *c, const sb_decode_plan *p)
{
    if (!c || !p) return fail("null argument");
    if (!p->layers || !p->n_layers || !p->hidden || !p->vocab || !p->ctx || !p->final_norm)
        return fail("decode plan: incomplete");
    if (p->ctx > (1u << 24)) return fail("decode plan: ctx too large");
    std::lock_guard<std::mutex> lk(c->mu);
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    if (c->eng) {
        cudaStreamSynchronize(c->stream);
        sb_engine_free(c->eng);
        c->eng = nullptr;
    }
    sb_engine *e = new sb_engine();
    auto bail = [&](int rc) {
        delete e;
        return rc;
    };
    e->H = p->hidden;
    e->V = p->vocab;
    e->ctx = p->ctx;
    e->eps = p->eps;
    sb_group *const g = (c->grp && c->grp->world > 1) ? c->grp : nullptr;
    if (g && !g->opened) return bail(fail("decode plan: the group is not open (sb_group_open)"));
    if (g && (p->hidden > (size_t)sb::grp::XW || 2 * p->n_layers + 1 > (size_t)sb::grp::NX)) return bail(0);
    e->tp = g;
    const size_t H = e->H;
    size_t attn_ws = 0;
    e->L.resize(p->n_layers);
    for (size_t l = 0; l < p->n_layers; l++) {
        const sb_layer_plan &lp = p->layers[l];
        EngLayer &L = e->L[l];
        if (!lp.norm_attn || !lp.norm_ffn) return bail(fail("decode plan: layer without norms"));
        L.heads = lp.heads, L.kvh = lp.kv_heads, L.hd = lp.head_dim, L.theta = lp.theta, L.neox = lp.neox;
        int rc;
        std::vector<float> tp_bias;  // this rank's slice of the q|k|v bias
        // tensor-parallel attention when the query heads split evenly and each rank's heads
        // read whole kv heads (or share one); else (and for MLA) every rank computes it whole
        size_t tp_hp = 0, tp_kvl = 0;
        if (g && !lp.mla && L.heads && L.kvh && L.heads % L.kvh == 0 && L.hd == 128 && L.heads % g->world == 0) {
            const size_t gs = L.heads / L.kvh, hp = L.heads / g->world;
            const size_t kvl = hp % gs == 0 ? hp / gs : gs % hp == 0 ? 1 : 0;
            if (kvl && hp / kvl <= 8) tp_hp = hp, tp_kvl = kvl;
        }
        if (lp.mla) {
            // MLA: latent cache + rope keys; attention output heads * v_dim wide
            const sb_mla_plan &ml = *lp.mla;
            L.mla = true, L.q_rank = ml.q_rank, L.kv_rank = ml.kv_rank, L.qk_nope = ml.qk_nope;
            L.qk_rope = ml.qk_rope, L.v_dim = ml.v_dim;
            if (!L.heads || !L.kvh || L.heads % L.kvh || L.heads > (size_t)sb::mla::MAXH || L.kv_rank % 512 ||
                L.kv_rank > (size_t)sb::mla::MAXR || !L.qk_nope || L.qk_nope > (size_t)sb::mla::AB_RG * sb::mla::AB_ROWS ||
                !L.qk_rope || L.qk_rope % 2 ||
                L.qk_rope > (size_t)sb::mla::MAXRP || !L.v_dim || !L.q_rank)
                return bail(0);
            const size_t qk = L.qk_nope + L.qk_rope;
            L.qd = L.heads * L.v_dim;  // attention output width
            if ((rc = eng_mat(c, ml.q_down, L.q_rank, H, &L.q_down, true)) != 1) return bail(rc);
            if ((rc = eng_mat(c, ml.q_up, L.heads * qk, L.q_rank, &L.q_up, true)) != 1) return bail(rc);
            if ((rc = eng_mat(c, ml.kv_down, L.kv_rank, H, &L.kv_down, true)) != 1) return bail(rc);
            if ((rc = eng_mat(c, ml.k_up, L.kvh * qk, L.kv_rank, &L.k_up, true)) != 1) return bail(rc);
            if ((rc = eng_mat(c, ml.v_up, L.kvh * L.v_dim, L.kv_rank, &L.v_up, true)) != 1) return bail(rc);
            if (L.k_up.dt != SB_DTYPE_Q4_K) return bail(0);  // the absorption reads Q4_K rows
            if ((rc = eng_mat(c, lp.o, H, L.qd, &L.o, true)) != 1) return bail(rc);
            L.latent = (uint16_t *)e->dalloc(e->ctx * L.kv_rank * 2, &err);
            if (err == cudaSuccess) L.krope = (float *)e->dalloc(e->ctx * L.kvh * L.qk_rope * 4, &err);
            if (err != cudaSuccess) return bail(fail("cudaMalloc(latent cache)", err));
            e->mla_q = std::max(e->mla_q, L.q_rank);
            e->mla_r = std::max(e->mla_r, L.kv_rank);
            e->mla_qq = std::max(e->mla_qq, L.heads * qk);
            e->mla_hr = std::max(e->mla_hr, L.heads * L.kv_rank);
            e->mla_hp = std::max(e->mla_hp, L.heads * L.qk_rope);
            e->mla_ws_bytes = std::max(e->mla_ws_bytes, sbk_mla_ws_bytes(L.heads, L.kv_rank));
        } else if (tp_hp) {
            // tensor-parallel attention: this rank's query heads, the kv heads they read, the
            // matching columns of attn_output (its partial sums go through the exchange)
            const size_t r = g->rank, gs = L.heads / L.kvh, hp = tp_hp, kvl = tp_kvl;
            L.tp_attn = true;
            const size_t q0 = r * hp, kv0 = q0 / gs, qdg = L.heads * L.hd, kvdg = L.kvh * L.hd;
            L.heads = hp, L.kvh = kvl, L.qd = hp * L.hd, L.kvd = kvl * L.hd;
            if ((rc = eng_mat_rows(c, lp.q, qdg, H, q0 * L.hd, L.qd, &L.q)) != 1) return bail(rc);
            if ((rc = eng_mat_rows(c, lp.k, kvdg, H, kv0 * L.hd, L.kvd, &L.k)) != 1) return bail(rc);
            if ((rc = eng_mat_rows(c, lp.v, kvdg, H, kv0 * L.hd, L.kvd, &L.v)) != 1) return bail(rc);
            if ((rc = eng_mat_cols(c, lp.o, H, qdg, q0 * L.hd, L.qd, &L.o)) != 1) return bail(rc);
            if (lp.qkv_bias) {
                const float *b0 = lp.qkv_bias;
                tp_bias.insert(tp_bias.end(), b0 + q0 * L.hd, b0 + q0 * L.hd + L.qd);
                tp_bias.insert(tp_bias.end(), b0 + qdg + kv0 * L.hd, b0 + qdg + kv0 * L.hd + L.kvd);
                tp_bias.insert(tp_bias.end(), b0 + qdg + kvdg + kv0 * L.hd, b0 + qdg + kvdg + kv0 * L.hd + L.kvd);
            }
        } else {
            if (!L.heads || !L.kvh || L.heads % L.kvh || L.hd != 128 || L.heads / L.kvh > 8) return bail(0);
            L.qd = L.heads * L.hd, L.kvd = L.kvh * L.hd;
            if ((rc = eng_mat(c, lp.q, L.qd, H, &L.q, true)) != 1) return bail(rc);
            if ((rc = eng_mat(c, lp.k, L.kvd, H, &L.k, true)) != 1) return bail(rc);
            if ((rc = eng_mat(c, lp.v, L.kvd, H, &L.v, true)) != 1) return bail(rc);
            if ((rc = eng_mat(c, lp.o, H, L.qd, &L.o, true)) != 1) return bail(rc);
        }
        if (lp.moe) {
            // MoE FFN: every expert resident, its tensor map in a device table
            const sb_moe_plan &mp = *lp.moe;
            if (!mp.n_exp || !mp.top_k || mp.top_k > mp.n_exp || mp.top_k > 16 || mp.n_exp > 1024 || !mp.experts ||
                !mp.ffn || mp.ffn % 32)
                return bail(0);
            L.moe = true, L.n_exp = mp.n_exp, L.top_k = mp.top_k, L.effn = mp.ffn;
            L.has_sh = mp.shared != nullptr;
            if (2 * (L.top_k + (L.has_sh ? 1 : 0)) > (size_t)sb::tcmv::MAXB ||
                L.top_k + (L.has_sh ? 1 : 0) > (size_t)sb::tcmv::XS_MAXY)
                return bail(0);
            if (g && L.top_k + 1 > (size_t)sb::grp::DSL) return bail(0);
            // the router on every rank; the experts resident here: all of them, or under
            // expert parallelism this rank's range of expert IDs (row_strip), and the shared
            // expert on rank l % world
            if (mp.router.view.dtype == SB_DTYPE_F32) {
                // an f32 router (as the reference stores it), one GPU only
                if (g || H * 4 > 48 * 1024) return bail(0);
                if (!mp.router.key || !mp.router.view.bytes || mp.router.view.len != L.n_exp * H * 4 ||
                    mp.router.rows != L.n_exp || mp.router.cols != H)
                    return bail(fail("decode plan: f32 router of an unexpected shape"));
                Resident *r = nullptr;
                if ((rc = c->resident(mp.router.key, &mp.router.view, L.n_exp, H, &r, false)) != 1) return bail(rc);
                L.router = EngMat{r->ptr, SB_DTYPE_F32, L.n_exp, H};
            } else if ((rc = eng_mat(c, mp.router, L.n_exp, H, &L.router, true)) != 1) {
                return bail(rc);
            }
            if (g) {
                int lo, hi;
                sb::row_strip((int)L.n_exp, g->rank, g->world, lo, hi);
                if (hi <= lo) return bail(0);
                L.ex_lo = (size_t)lo, L.ex_hi = (size_t)hi;
                L.sh_here = L.has_sh && l % g->world == (size_t)g->rank;
            } else {
                L.ex_lo = 0, L.ex_hi = L.n_exp;
                L.sh_here = L.has_sh;
            }
            const size_t nl = L.ex_hi - L.ex_lo;
            L.ex.resize(3 * nl);
            std::vector<CUtensorMap> maps(3 * nl);
            // gate and up of each expert as one matrix of 16-row group pairs (its launch forms
            // silu(gate) * up) when both are of one tensor-core format
            {
                auto pairable = [&](const sb_mat &g, const sb_mat &u, size_t f) {
                    const uint8_t dt = g.view.dtype;
                    return g.view.bytes && u.view.bytes && dt == u.view.dtype && f % 16 == 0 &&
                           (dt == SB_DTYPE_Q4_K || dt == SB_DTYPE_Q6_K || dt == SB_DTYPE_Q8_0);
                };
                L.ex_pairs = pairable(mp.experts[3 * L.ex_lo], mp.experts[3 * L.ex_lo + 1], L.effn) &&
                             (!L.sh_here || pairable(mp.shared[0], mp.shared[1], mp.shared[0].rows));
            }
            for (size_t x = 0; x < nl; x++) {
                const size_t r[3] = {L.effn, L.effn, H}, cc[3] = {H, H, L.effn};
                for (int k = 0; k < 3; k++) {
                    EngMat &m = L.ex[3 * x + k];
                    if (L.ex_pairs && k == 1) {  // (the pair matrix's slot repeated)
                        m = L.ex[3 * x];
                        maps[3 * x + 1] = maps[3 * x];
                        continue;
                    }
                    if (L.ex_pairs && k == 0) {
                        const sb_mat &eg = mp.experts[3 * (L.ex_lo + x)], &eu = mp.experts[3 * (L.ex_lo + x) + 1];
                        if ((rc = eng_mat_pairs(c, eg, eu, L.effn, H, 0, L.effn, &m)) != 1) return bail(rc);
                    } else if ((rc = eng_mat(c, mp.experts[3 * (L.ex_lo + x) + k], r[k], cc[k], &m, true)) != 1) {
                        return bail(rc);
                    }
                    if (m.dt != L.ex[k].dt) return bail(0);  // one dtype per matrix kind
                    const int mr =
                        m.dt == SB_DTYPE_Q4_K
                            ? sb::tcmv::make_map<sb::tcmv::Q4K>(&maps[3 * x + k], m.w, (int)m.rows, (int)m.cols)
                        : m.dt == SB_DTYPE_Q6_K_P
                            ? sb::tcmv::make_map<sb::tcmv::Q6KP>(&maps[3 * x + k], m.w, (int)m.rows, (int)m.cols)
                        : (m.dt == SB_DTYPE_Q8_0_R || (m.dt == SB_DTYPE_Q8_0 && m.cols % 128 == 0)) && k == 2
                            ? sb::tcmv::make_map<sb::tcmv::Q80>(&maps[3 * x + k], m.w, (int)m.rows, (int)m.cols)
                            : 1;
                    if (mr > 0) return bail(0);  // expert dtype without a tensor-core kernel
                    if (mr < 0) return bail(fail("decode plan: tensor map of an expert rejected"));
                }
            }
            if (L.has_sh && !L.sh_here) {
                if (upload_f32(e, mp.shared_gate, H, &L.sg)) return bail(-1);
            } else if (L.has_sh) {
                L.sffn = mp.shared[0].rows;
                const size_t r[3] = {L.sffn, L.sffn, H}, cc[3] = {H, H, L.sffn};
                for (int k = 0; k < 3; k++) {
                    if (L.ex_pairs && k == 1) {
                        L.sh[1] = L.sh[0];
                        continue;
                    }
                    if (L.ex_pairs && k == 0)
                        rc = eng_mat_pairs(c, mp.shared[0], mp.shared[1], L.sffn, H, 0, L.sffn, &L.sh[0]);
                    else
                        rc = eng_mat(c, mp.shared[k], r[k], cc[k], &L.sh[k], true);
                    if (rc != 1) return bail(rc);
                    if (L.sh[k].dt != L.ex[k].dt) return bail(0);
                }
                if (upload_f32(e, mp.shared_gate, H, &L.sg)) return bail(-1);
            }
            L.maps = (CUtensorMap *)e->dalloc(maps.size() * sizeof(CUtensorMap), &err);
            if (err != cudaSuccess) return bail(fail("cudaMalloc(tensor maps)", err));
            if ((err = cudaMemcpy(L.maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice)) !=
                cudaSuccess)
                return bail(fail("cudaMemcpy(tensor maps)", err));
            e->moe_slots = std::max(e->moe_slots, L.top_k + (L.has_sh ? 1 : 0));
            e->moe_ffn = std::max(e->moe_ffn, std::max(L.effn, L.sffn));
            e->n_exp_max = std::max(e->n_exp_max, L.n_exp);
        } else if (g && lp.gate.rows % 256 == 0 && lp.gate.rows / 256 >= (size_t)g->world) {
            // tensor-parallel FFN: whole 256-column blocks of the intermediate dimension per
            // rank (other widths: every rank computes the FFN whole)
            const size_t ffn_g = lp.gate.rows;
            int b0, b1;
            sb::row_strip((int)(ffn_g / 256), g->rank, g->world, b0, b1);
            L.tp_ffn = true;
            const size_t f0 = 256 * (size_t)b0;
            L.ffn = 256 * (size_t)(b1 - b0);
            if ((rc = eng_mat_pairs(c, lp.gate, lp.up, ffn_g, H, f0, L.ffn, &L.gu2)) < 0) return bail(rc);
            if (rc != 1 && (rc = eng_mat_rows(c, lp.gate, ffn_g, H, f0, L.ffn, &L.g)) != 1) return bail(rc);
            if (!L.gu2.w && (rc = eng_mat_rows(c, lp.up, ffn_g, H, f0, L.ffn, &L.u)) != 1) return bail(rc);
            if ((rc = eng_mat_cols(c, lp.down, H, ffn_g, f0, L.ffn, &L.d)) != 1) return bail(rc);
        } else {
            L.ffn = lp.gate.rows;
            if ((rc = eng_mat_pairs(c, lp.gate, lp.up, L.ffn, H, 0, L.ffn, &L.gu2)) < 0) return bail(rc);
            if (rc != 1 && (rc = eng_mat(c, lp.gate, L.ffn, H, &L.g, true)) != 1) return bail(rc);
            if (!L.gu2.w && (rc = eng_mat(c, lp.up, L.ffn, H, &L.u, true)) != 1) return bail(rc);
            if ((rc = eng_mat(c, lp.down, H, L.ffn, &L.d, true)) != 1) return bail(rc);
        }
        if (lp.rope_factors && (L.mla || !(lp.rope_mscale > 0.0f) || !std::isfinite(lp.rope_mscale)))
            return bail(0);  // YaRN on GQA layers only, with a positive mscale
        L.rms = lp.rope_factors ? lp.rope_mscale : 1.0f;
        if (upload_f32(e, lp.norm_attn, H, &L.na) || upload_f32(e, lp.norm_ffn, H, &L.nf) ||
            upload_f32(e, lp.rope_factors, L.hd / 2, &L.rf) ||
            upload_f32(e, lp.q_norm, L.hd, &L.qn) || upload_f32(e, lp.k_norm, L.hd, &L.kn) ||
            upload_f32(e, L.tp_attn ? (tp_bias.empty() ? nullptr : tp_bias.data()) : lp.qkv_bias, L.qd + 2 * L.kvd,
                       &L.bias))
            return bail(-1);
        if (L.mla) {
            e->kv_rows_total += L.kv_rank;
            e->qkv_max = std::max(e->qkv_max, L.qd);
        } else {
            L.kc = (uint16_t *)e->dalloc(e->ctx * L.kvd * 2, &err);
            if (err == cudaSuccess) L.vc = (uint16_t *)e->dalloc(e->ctx * L.kvd * 2, &err);
            if (err != cudaSuccess) return bail(fail("cudaMalloc(kv cache)", err));
            e->qkv_max = std::max(e->qkv_max, L.qd + 2 * L.kvd);
            e->kv_rows_total += 2 * L.kvd;
            attn_ws = std::max(attn_ws, sbk_attn_ws_bytes(L.heads, L.kvh, L.hd, e->ctx));
        }
        e->ffn_max = std::max(e->ffn_max, L.ffn);
    }
    int rc;
    if (g) {  // this rank's rows of the output matrix
        int v0, v1;
        sb::row_strip((int)e->V, g->rank, g->world, v0, v1);
        e->vbase = (size_t)v0, e->vn = (size_t)(v1 - v0);
        if ((rc = eng_mat_rows(c, p->lm_head, e->V, H, e->vbase, e->vn, &e->lm)) != 1) return bail(rc);
    } else {
        e->vbase = 0, e->vn = e->V;
        if ((rc = eng_mat(c, p->lm_head, e->V, H, &e->lm, true)) != 1) return bail(rc);
    }
    if (p->embed.view.bytes) {
        if (!sbk_row_bytes(p->embed.view.dtype, H) && p->embed.view.dtype != SB_DTYPE_F32) return bail(0);
        if ((rc = eng_mat(c, p->embed, e->V, H, &e->emb, false)) != 1) return bail(rc);
    }
    if (upload_f32(e, p->final_norm, H, &e->fnorm)) return bail(-1);
    // activations (each padded to 64 floats)
    auto fbuf = [&](size_t n) { return (float *)e->dalloc(((n + 63) & ~(size_t)63) * 4, &err); };
    e->h = fbuf(H);
    e->h2 = fbuf(H);
    e->qkv = fbuf(e->qkv_max);
    e->att = fbuf(e->qkv_max);
    e->ob = fbuf(H);
    e->gu = fbuf(2 * e->ffn_max);
    e->tmp = fbuf(std::max(e->ffn_max, std::max(H, e->qkv_max)));
    e->logits = fbuf(e->V);
    if (e->moe_slots) {
        e->rlog = fbuf(e->n_exp_max);
        e->wts = fbuf(e->moe_slots);
        e->ridx = (int *)fbuf(e->moe_slots);
        e->rtrace = (int *)fbuf(e->ctx * e->L.size() * sb::RT_W);  // top_k <= 16 (checked above)
        e->moe_ffn = (e->moe_ffn + 63) & ~(size_t)63;
        e->egu = fbuf(2 * e->moe_slots * e->moe_ffn);
        e->ys = fbuf(e->moe_slots * H);
    }
    if (e->mla_r) {
        e->mcq = fbuf(e->mla_q);
        e->mc = fbuf(e->mla_r);
        e->mq = fbuf(e->mla_qq);
        e->mqt = fbuf(e->mla_hr);
        e->mqr = fbuf(e->mla_hp);
        e->mcbar = fbuf(e->mla_hr);
        e->mla_ws = e->dalloc(e->mla_ws_bytes, &err);
    }
    e->ints = (int *)e->dalloc(64, &err);
    e->prompt = (int *)e->dalloc(e->ctx * 4, &err);
    e->hist = (int *)e->dalloc(e->ctx * 4, &err);
    e->attn_ws = e->dalloc(attn_ws, &err);
    e->am_ws = e->dalloc(sbk_argmax_ws_bytes(), &err);
    e->kv_rows = (uint16_t *)e->dalloc(e->kv_rows_total * 2, &err);
    {
        std::vector<sb::KvSeg> segs;
        long long o = 0;
        for (auto &L : e->L) {
            if (L.mla) {
                segs.push_back(sb::KvSeg{L.latent, o, (int)L.kv_rank, 0});
                o += (long long)L.kv_rank;
            } else {
                segs.push_back(sb::KvSeg{L.kc, o, (int)L.kvd, 0});
                segs.push_back(sb::KvSeg{L.vc, o + (long long)L.kvd, (int)L.kvd, 0});
                o += 2 * (long long)L.kvd;
            }
        }
        e->n_kv_segs = segs.size();
        e->kv_segs = e->dalloc(segs.size() * sizeof(sb::KvSeg), &err);
        if (err != cudaSuccess) return bail(fail("cudaMalloc(kv segments)", err));
        if ((err = cudaMemcpy(e->kv_segs, segs.data(), segs.size() * sizeof(sb::KvSeg), cudaMemcpyHostToDevice)) !=
            cudaSuccess)
            return bail(fail("cudaMemcpy(kv segments)", err));
    }
    // zeroed state; one eager token of each kind (sets kernel attributes, builds the MoE
    // batches, creates the per-stream matvec workspace outside any capture), then capture,
    // then re-zero.  With a tensor-parallel group the warm-up token exchanges with the other
    // ranks, so it waits for sb_decode_finish (called on every rank after a host barrier).
    e->attn_ws_bytes = attn_ws;
    if (g) {
        e->pending_finish = true;
        c->eng = e;
        return 1;
    }
    if ((err = engine_zero(e, c->stream)) != cudaSuccess) return bail(fail("decode state reset", err));
    if ((rc = enqueue_token(e, c->stream, false))) return bail(rc);
    if (e->emb.w && (rc = enqueue_token(e, c->stream, true))) return bail(rc);
    if ((err = cudaStreamSynchronize(c->stream)) != cudaSuccess) return bail(fail("decode warm-up", err));
    if ((rc = capture(e, c->stream, false, &e->g_tok))) return bail(rc);
    if (e->emb.w && (rc = capture(e, c->stream, true, &e->g_greedy))) return bail(rc);
    if ((err = engine_zero(e, c->stream)) != cudaSuccess) return bail(fail("decode state reset", err));
    c->eng = e;
    return 1;
}

extern "C" int sb_decode_finish(sb_ctx *c)
{
    if (!c) return fail("null context");
    std::lock_guard<std::mutex> lk(c->mu);
    sb_engine *e = c->eng;
    if (!e) return 0;
    if (!e->pending_finish) return 1;
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    int rc;
    if ((err = engine_zero(e, c->stream)) != cudaSuccess) return fail("decode state reset", err);
    if (!e->emb.w) return fail("sb_decode_finish: a tensor-parallel engine needs the embedding table");
    if ((rc = enqueue_token(e, c->stream, true))) return rc;
    if ((err = cudaStreamSynchronize(c->stream)) != cudaSuccess) return fail("decode warm-up", err);
    if ((rc = capture(e, c->stream, true, &e->g_greedy))) return rc;
    if ((err = engine_zero(e, c->stream)) != cudaSuccess) return fail("decode state reset", err);
    e->pending_finish = false;
    return 1;
}

extern "C" int sb_decode_token(sb_ctx *c, const float *embed, size_t pos, float *logits, uint16_t *kv_rows)
{
    if (!c) return fail("null context");
    if (!embed || !logits) return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    sb_engine *e = c->eng;
    if (!e || !e->g_tok || e->tp) return 0;  // a tensor-parallel engine holds a slice of the logits
    if (pos >= e->ctx) return fail("sb_decode_token: position beyond the prepared context");
    const uint64_t t0 = now_ns();
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    const size_t hb = (e->H * 4 + 255) & ~(size_t)255, lb = (e->V * 4 + 255) & ~(size_t)255;
    if (c->ensure_host_stage(hb + 256 + lb + e->kv_rows_total * 2)) return -1;
    char *hs = (char *)c->host_stage;
    memcpy(hs, embed, e->H * 4);
    *(int *)(hs + hb) = (int)pos;
    if ((err = cudaMemcpyAsync(e->h, hs, e->H * 4, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess ||
        (err = cudaMemcpyAsync(e->ints, hs + hb, 4, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(decode input)", err);
    if ((err = cudaGraphLaunch(e->g_tok, c->stream)) != cudaSuccess) return fail("cudaGraphLaunch", err);
    if ((err = cudaMemcpyAsync(hs + hb + 256, e->logits, e->V * 4, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(logits)", err);
    if (kv_rows && (err = cudaMemcpyAsync(hs + hb + 256 + lb, e->kv_rows, e->kv_rows_total * 2,
                                          cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(kv rows)", err);
    if ((err = cudaStreamSynchronize(c->stream)) != cudaSuccess) return fail("cudaStreamSynchronize", err);
    std::vector<HostCopy> cp{HostCopy{logits, hs + hb + 256, e->V * 4}};
    if (kv_rows) cp.push_back(HostCopy{kv_rows, hs + hb + 256 + lb, e->kv_rows_total * 2});
    c->copy(cp);
    e->last_pos = pos, e->traced = true;
    c->stats.launches += e->launches_per_token;
    c->stats.bytes_up += e->H * 4 + 4;
    c->stats.bytes_down += e->V * 4 + (kv_rows ? e->kv_rows_total * 2 : 0);
    c->stats.decode_embed_up += e->H * 4;
    c->stats.decode_control_up += 4;
    c->stats.decode_logits_down += e->V * 4;
    c->stats.decode_kv_down += kv_rows ? e->kv_rows_total * 2 : 0;
    c->stats.decode_steps += 1;
    c->stats.total_ns += now_ns() - t0;
    return 1;
}

extern "C" int sb_decode_greedy(sb_ctx *c, const int32_t *prompt, size_t n_prompt, size_t pos, size_t n,
                                int32_t *tokens_out)
{
    if (!c) return fail("null context");
    if (!prompt || !n_prompt || !tokens_out) return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    sb_engine *e = c->eng;
    if (e && e->pending_finish) return fail("sb_decode_greedy: call sb_decode_finish first (tensor-parallel group)");
    if (!e || !e->g_greedy) return 0;
    if (n == 0) return 1;
    if (pos + n > e->ctx || n_prompt > e->ctx) return fail("sb_decode_greedy: beyond the prepared context");
    for (size_t i = 0; i < n_prompt; i++)
        if (prompt[i] < 0 || (size_t)prompt[i] >= e->V) return fail("sb_decode_greedy: token id out of range");
    const uint64_t t0 = now_ns();
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    const size_t pb = (n_prompt * 4 + 255) & ~(size_t)255;
    if (c->ensure_host_stage(pb + 256 + n * 4)) return -1;
    char *hs = (char *)c->host_stage;
    memcpy(hs, prompt, n_prompt * 4);
    int *ints = (int *)(hs + pb);
    ints[0] = (int)pos, ints[1] = prompt[0], ints[2] = 0, ints[3] = (int)n_prompt;
    if ((err = cudaMemcpyAsync(e->prompt, hs, n_prompt * 4, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess ||
        (err = cudaMemcpyAsync(e->ints, ints, 16, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(greedy input)", err);
    for (size_t i = 0; i < n; i++)
        if ((err = cudaGraphLaunch(e->g_greedy, c->stream)) != cudaSuccess) return fail("cudaGraphLaunch", err);
    if ((err = cudaMemcpyAsync(hs + pb + 256, e->hist, n * 4, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess)
        return fail("cudaMemcpyAsync(tokens)", err);
    if ((err = cudaStreamSynchronize(c->stream)) != cudaSuccess) return fail("cudaStreamSynchronize", err);
    memcpy(tokens_out, hs + pb + 256, n * 4);
    e->last_pos = pos + n - 1, e->traced = true;
    c->stats.launches += e->launches_per_token * n;
    c->stats.bytes_up += n_prompt * 4 + 16;
    c->stats.bytes_down += n * 4;
    c->stats.decode_control_up += n_prompt * 4 + 16;
    c->stats.decode_steps += n;
    c->stats.total_ns += now_ns() - t0;
    return 1;
}

namespace sb {
// f16 rows -> f32 (exact), for re-forming an MLA layer's rope keys from uploaded latent rows.
__global__ void f16_to_f32_kernel(const uint16_t *__restrict__ src, float *__restrict__ dst, int n)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) dst[i] = f16_to_f32(src[i]);
}
}  // namespace sb

extern "C" int sb_decode_upload_state(sb_ctx *c, const sb_layer_state *layers, size_t n_layers, size_t pos)
{
    if (!c) return fail("null context");
    if (!layers) return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    sb_engine *e = c->eng;
    if (!e || e->tp || e->pending_finish) return 0;
    if (n_layers != e->L.size()) return fail("sb_decode_upload_state: layer count differs from the plan's");
    if (pos > e->ctx) return fail("sb_decode_upload_state: position beyond the prepared context");
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    const uint64_t t0 = now_ns();
    int *tpos = nullptr;  // positions 0 .. pos-1 of the MLA rows to re-form
    bool any_mla = false;
    for (size_t l = 0; l < n_layers; l++) {
        const sb_layer_state &st = layers[l];
        const EngLayer &L = e->L[l];
        if (!st.valid_rows || !st.k || (!L.mla && !st.v)) return fail("sb_decode_upload_state: layer without rows");
        any_mla |= L.mla && std::min(*st.valid_rows, pos) < pos;
    }
    if (any_mla) {
        std::vector<int> h(pos);
        for (size_t t = 0; t < pos; t++) h[t] = (int)t;
        if ((err = cudaMalloc(&tpos, std::max<size_t>(pos, 1) * 4)) != cudaSuccess) return fail("cudaMalloc", err);
        if ((err = cudaMemcpy(tpos, h.data(), pos * 4, cudaMemcpyHostToDevice)) != cudaSuccess) {
            cudaFree(tpos);
            return fail("cudaMemcpy", err);
        }
    }
    auto done = [&](int rc) {
        if (tpos) {
            cudaStreamSynchronize(c->stream);
            cudaFree(tpos);
        }
        return rc;
    };
    for (size_t l = 0; l < n_layers; l++) {
        const sb_layer_state &st = layers[l];
        EngLayer &L = e->L[l];
        const size_t v0 = std::min(*st.valid_rows, pos);
        if (v0 < pos) {
            const size_t w = L.mla ? L.kv_rank : L.kvd;  // f16 values a row
            uint16_t *kd = L.mla ? L.latent : L.kc;
            if ((err = cudaMemcpyAsync(kd + v0 * w, st.k + v0 * w, (pos - v0) * w * 2, cudaMemcpyHostToDevice,
                                       c->stream)) != cudaSuccess)
                return done(fail("cudaMemcpyAsync(k rows)", err));
            if (!L.mla && (err = cudaMemcpyAsync(L.vc + v0 * w, st.v + v0 * w, (pos - v0) * w * 2,
                                                 cudaMemcpyHostToDevice, c->stream)) != cudaSuccess)
                return done(fail("cudaMemcpyAsync(v rows)", err));
            c->stats.bytes_up += (pos - v0) * w * (L.mla ? 2 : 4);
            if (L.mla) {
                // the absorb step of each row again, on its own latent row (f16 -> f32 -> f16 is
                // exact, so the cache keeps its bits): the row's rope keys as the step formed them
                if ((err = cudaMemsetAsync(e->mq, 0, L.heads * (L.qk_nope + L.qk_rope) * 4, c->stream)) != cudaSuccess)
                    return done(fail("cudaMemsetAsync", err));
                for (size_t t = v0; t < pos; t++) {
                    sb::f16_to_f32_kernel<<<1, 512, 0, c->stream>>>(L.latent + t * L.kv_rank, e->mc, (int)L.kv_rank);
                    if ((err = cudaGetLastError()) != cudaSuccess) return done(fail("f16 rows launch", err));
                    const int rc = sbk_mla_absorb(e->mq, e->mc, L.k_up.w, L.k_up.dt, L.latent, L.krope, e->mqt, e->mqr,
                                                  tpos + t, L.heads, L.kvh, L.kv_rank, L.qk_nope, L.qk_rope, e->ctx,
                                                  L.theta, 0, c->stream);
                    if (rc) return done(fail("sbk_mla_absorb (state upload) failed (" + std::to_string(rc) + ")"));
                    c->stats.launches += 2;
                }
            }
        }
    }
    if ((err = cudaStreamSynchronize(c->stream)) != cudaSuccess) return done(fail("state upload", err));
    for (size_t l = 0; l < n_layers; l++) *layers[l].valid_rows = pos;
    c->stats.total_ns += now_ns() - t0;
    return done(1);
}

extern "C" int sb_decode_download_state(sb_ctx *c, const sb_layer_rows *layers, size_t n_layers, size_t rows,
                                        float *hidden)
{
    if (!c) return fail("null context");
    if (!layers && n_layers) return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    sb_engine *e = c->eng;
    if (!e || e->tp || e->pending_finish) return 0;
    if (n_layers != e->L.size()) return fail("sb_decode_download_state: layer count differs from the plan's");
    if (rows > e->ctx) return fail("sb_decode_download_state: more rows than the prepared context");
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    const uint64_t t0 = now_ns();
    for (size_t l = 0; l < n_layers; l++) {
        const EngLayer &L = e->L[l];
        const size_t w = L.mla ? L.kv_rank : L.kvd;
        if (!layers[l].k || (!L.mla && !layers[l].v)) return fail("sb_decode_download_state: layer without rows");
        if (!rows) continue;
        if ((err = cudaMemcpyAsync(layers[l].k, L.mla ? L.latent : L.kc, rows * w * 2, cudaMemcpyDeviceToHost,
                                   c->stream)) != cudaSuccess)
            return fail("cudaMemcpyAsync(k rows)", err);
        if (!L.mla && (err = cudaMemcpyAsync(layers[l].v, L.vc, rows * w * 2, cudaMemcpyDeviceToHost, c->stream)) !=
                          cudaSuccess)
            return fail("cudaMemcpyAsync(v rows)", err);
        c->stats.bytes_down += rows * w * (L.mla ? 2 : 4);
    }
    if (hidden) {
        if ((err = cudaMemcpyAsync(hidden, e->hfin, e->H * 4, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess)
            return fail("cudaMemcpyAsync(hidden)", err);
        c->stats.bytes_down += e->H * 4;
    }
    if ((err = cudaStreamSynchronize(c->stream)) != cudaSuccess) return fail("state download", err);
    c->stats.total_ns += now_ns() - t0;
    return 1;
}

namespace sb {
// Row `pos` of the route trace: the chosen IDs of every MoE layer (layer order, rank order)
// into idx, and when gaps != null the router-logit gap of each MoE layer into gaps.
static int read_route_row(sb_ctx *c, sb_engine *e, size_t pos, int32_t *idx, size_t n, float *gaps, size_t n_gaps,
                          const char *who)
{
    size_t need = 0, moe = 0;
    for (auto &L : e->L) need += L.moe ? L.top_k : 0, moe += L.moe ? 1 : 0;
    if (n < need) return fail(std::string(who) + ": output shorter than the MoE layers' choices");
    if (gaps && n_gaps < moe) return fail(std::string(who) + ": gap output shorter than the MoE layers");
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    const size_t row = e->L.size() * RT_W;
    std::vector<int> t(row);
    if ((err = cudaMemcpyAsync(t.data(), e->rtrace + pos * row, row * 4, cudaMemcpyDeviceToHost, c->stream)) !=
            cudaSuccess ||
        (err = cudaStreamSynchronize(c->stream)) != cudaSuccess)
        return fail(who, err);
    size_t o = 0, g = 0;
    for (size_t l = 0; l < e->L.size(); l++) {
        if (!e->L[l].moe) continue;
        for (size_t r = 0; r < e->L[l].top_k; r++) idx[o++] = t[l * RT_W + r];
        if (gaps) {
            int b = t[l * RT_W + RT_GAP];
            float f;
            memcpy(&f, &b, 4);
            gaps[g++] = f;
        }
    }
    return 1;
}
}  // namespace sb

extern "C" int sb_decode_routes(sb_ctx *c, int32_t *idx, size_t n)
{
    if (!c) return fail("null context");
    if (!idx) return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    sb_engine *e = c->eng;
    if (!e || !e->rtrace || !e->traced) return 0;
    return sb::read_route_row(c, e, e->last_pos, idx, n, nullptr, 0, "sb_decode_routes");
}

extern "C" int sb_decode_route_trace(sb_ctx *c, size_t pos, int32_t *idx, size_t n, float *gaps, size_t n_gaps)
{
    if (!c) return fail("null context");
    if (!idx) return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    sb_engine *e = c->eng;
    if (!e || !e->rtrace || !e->traced) return 0;
    if (pos >= e->ctx) return fail("sb_decode_route_trace: position beyond the prepared context");
    return sb::read_route_row(c, e, pos, idx, n, gaps, n_gaps, "sb_decode_route_trace");
}
