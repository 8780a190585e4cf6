// prefill_engine.cuh -- block prefill of a prompt through the whole-token engine's model:
// n tokens at positions pos0 .. pos0 + n - 1, layer by layer, every matrix product a
// tensor-core GEMM over all n tokens (pgemm.cuh), the steps between them over all rows
// (block.cuh).  The reference's block prefill: Runtime's prompt path over
// forward_layer_block (crates/soso-llm-core/src/layer.rs:1433) with its GPU offload
// (GpuDispatch::matmul / expertos_bloque / router_topk / atencion_prefill,
// crates/soso-llm-core/src/gpu.rs:443-530), then the logits of the last token
// (runtime.rs:1976-2019).
//
// The KV caches (f16 rows; MLA latent rows and rope keys) of those positions are filled
// exactly where the decode step would have put them, so decoding goes on at pos0 + n.
//
// Per layer (GQA):  x = rmsnorm(h) (f16) -> q|k|v GEMM -> bias / QK-norm / RoPE / K,V rows
//   -> causal attention -> o GEMM (the residual add goes into the next norm);
// (MLA): q_down|kv_down GEMM -> latent rows -> q_up GEMM; k_up and v_up GEMMs over every
//   cached latent row (the re-expansion of attention_decode_mla_latent, attn.rs:306-404,
//   for the whole block at once) -> RoPE of the rope slices (and the rope-key cache) ->
//   causal attention -> o GEMM;
// FFN (dense): x = rmsnorm(h + y) -> gate|up pair GEMM whose epilogue forms silu(g) * u
//   -> down GEMM;
// FFN (MoE): router GEMM -> top-k of every token -> pairs grouped by expert (tile tables
//   on the device) -> gathered inputs -> one grouped gate|up GEMM over every routed
//   expert -> one grouped down GEMM -> shared expert -> combine in choice order + residual.
// GEMM operands are f16 (the precision of the reference's f16 mma.sync prefill), sums f32.
#pragma once
#include <map>
#include <tuple>

#include "block.cuh"

extern "C" int sbk_matvec_batch(uint8_t dtype, const sbk_mv_op *ops, size_t n, int pdl, void *stream);

namespace pg = sb::pg;
namespace blk = sb::blk;

namespace {

// device buffers of the block prefill, for up to `cap` tokens
struct PfState {
    size_t cap = 0;
    std::vector<void *> allocs;
    int *tok = nullptr;
    float *h0 = nullptr, *h1 = nullptr, *y = nullptr, *x32 = nullptr, *qkv = nullptr, *att = nullptr;
    __half *x16 = nullptr, *att16 = nullptr, *act16 = nullptr;
    // MLA
    float *cq = nullptr, *c = nullptr, *q = nullptr, *kexp = nullptr;
    __half *cq16 = nullptr;
    uint16_t *k16 = nullptr, *v16 = nullptr;
    // MoE
    float *rlog = nullptr, *wts = nullptr, *yd = nullptr, *ysh = nullptr, *act32 = nullptr;
    int *idx = nullptr, *pair_slot = nullptr, *slot_tok = nullptr, *ntile = nullptr;
    __half *xg16 = nullptr, *actg16 = nullptr, *acts16 = nullptr;
    pg::Tile *t_gu = nullptr, *t_dn = nullptr;
    int cap_gu = 0, cap_dn = 0;
    // tile tables of the dense launches (rebuilt per call) and the per-launch descriptors
    pg::Tile *tiles = nullptr;
    size_t tiles_cap = 0;
    // per (matrix pointer): weight map in prefill form, and the Out descriptor tables
    CUtensorMap *maps = nullptr;
    size_t maps_cap = 0, maps_n = 0;
    std::map<const void *, int> map_of;
    std::map<const void *, int> blocks;  // contiguous map blocks (a layer's experts), by first matrix
    pg::Out *outs = nullptr;
    size_t outs_cap = 0, outs_n = 0;
    std::map<std::tuple<const void *, int, int, int>, CUtensorMap> xmaps;

    ~PfState()
    {
        for (void *p : allocs) cudaFree(p);
    }
    void *alloc(size_t bytes, cudaError_t *e)
    {
        void *p = nullptr;
        *e = cudaMalloc(&p, bytes ? bytes : 16);
        if (*e == cudaSuccess) allocs.push_back(p);
        return p;
    }
};

constexpr int PF_BN_SMALL = 64, PF_BN_LARGE = 256;

// formats of the dense GEMM launches (Q6_K as repacked for the matvec, four maps a matrix),
// and of the grouped expert launches (one map an expert)
bool pf_gemm_dtype(uint8_t dt)
{
    return dt == SB_DTYPE_Q4_K || dt == SB_DTYPE_Q8_0_R || dt == SB_DTYPE_Q8_0 || dt == SB_DTYPE_Q6_K_P;
}
bool pf_group_dtype(uint8_t dt) { return dt == SB_DTYPE_Q4_K || dt == SB_DTYPE_Q8_0_R || dt == SB_DTYPE_Q8_0; }

}  // namespace

void sb_pf_free(void *p) { delete reinterpret_cast<PfState *>(p); }

namespace {

// Token tile width.  A tile's time is set by dequantising its 128 x K weights (the same for
// both widths); the small tile fits two CTAs an SM, the large one takes ~1.5x as long (four
// times the MMAs and X) but dequantises each weight once per 256 tokens instead of 64.  Take
// the width whose waves of tiles end first.
int pick_bn(int rows_total, int ntok, int sms)
{
    const int rt = (rows_total + pg::BM - 1) / pg::BM;
    const int w64 = (rt * ((ntok + PF_BN_SMALL - 1) / PF_BN_SMALL) + 2 * sms - 1) / (2 * sms);
    const int w256 = (rt * ((ntok + PF_BN_LARGE - 1) / PF_BN_LARGE) + sms - 1) / sms;
    return 3 * w256 < 2 * w64 ? PF_BN_LARGE : PF_BN_SMALL;
}

// Grow the prefill buffers to n tokens (all sized from the engine's plan).
int pf_state(sb_ctx *c, sb_engine *e, size_t n, PfState **out)
{
    PfState *st = reinterpret_cast<PfState *>(e->pf);
    if (st && st->cap >= n) {
        *out = st;
        return 0;
    }
    const size_t cap = std::max<size_t>(n, st ? 2 * st->cap : 64);
    if (st) {
        cudaStreamSynchronize(c->stream);
        delete st;
        e->pf = nullptr;
    }
    st = new PfState();
    st->cap = cap;
    cudaError_t err = cudaSuccess;
    const size_t H = e->H;
    size_t qkv_w = 0, qd = 0, ffn = 0, qr = 0, kr = 0, mq = 0, kx = 0, vx = 0, nexp = 0, topk = 0, effn = 0, sffn = 0;
    bool sg = false;
    for (auto &L : e->L) {
        if (L.mla) {
            qr = std::max(qr, L.q_rank), kr = std::max(kr, L.kv_rank);
            mq = std::max(mq, L.heads * (L.qk_nope + L.qk_rope));
            kx = std::max(kx, L.kvh * (L.qk_nope + L.qk_rope)), vx = std::max(vx, L.kvh * L.v_dim);
            qd = std::max(qd, L.heads * L.v_dim);
        } else {
            qkv_w = std::max(qkv_w, L.qd + 2 * L.kvd), qd = std::max(qd, L.qd);
        }
        if (L.moe) {
            nexp = std::max(nexp, L.n_exp), topk = std::max(topk, L.top_k), effn = std::max(effn, L.effn);
            if (L.sh_here) sffn = std::max(sffn, L.sh[0].rows / 2);
            sg |= L.sg != nullptr || L.router.dt == SB_DTYPE_F32;  // (x32: shared gate, f32 router)
        } else {
            ffn = std::max(ffn, L.ffn);
        }
    }
    auto F = [&](size_t count) { return (float *)st->alloc(count * 4, &err); };
    auto Hh = [&](size_t count) { return (__half *)st->alloc(count * 2, &err); };
    st->tok = (int *)st->alloc(cap * 4, &err);
    st->h0 = F(cap * H), st->h1 = F(cap * H), st->y = F(cap * H), st->x16 = Hh(cap * H);
    if (sg) st->x32 = F(cap * H);
    if (qkv_w) st->qkv = F(cap * qkv_w);
    if (qd) st->att = F(cap * qd), st->att16 = Hh(cap * qd);
    if (ffn) st->act16 = Hh(cap * ffn), st->act32 = F(cap * ffn);
    if (kr) {
        st->cq = F(cap * qr), st->cq16 = Hh(cap * qr), st->c = F(cap * kr), st->q = F(cap * mq);
        st->kexp = F(e->ctx * kx), st->k16 = (uint16_t *)Hh(e->ctx * kx), st->v16 = (uint16_t *)Hh(e->ctx * vx);
    }
    if (nexp) {
        const size_t np = cap * topk;
        st->rlog = F(cap * nexp), st->wts = F(cap * topk), st->yd = F(np * H);
        st->idx = (int *)st->alloc(cap * topk * 4, &err), st->pair_slot = (int *)st->alloc(np * 4, &err);
        st->slot_tok = (int *)st->alloc(np * 4, &err), st->ntile = (int *)st->alloc(64, &err);
        st->xg16 = Hh(np * H), st->actg16 = Hh(np * effn);
        if (sffn) st->acts16 = Hh(cap * sffn), st->ysh = F(cap * H);
        // tiles: per expert (rows / 128) x (its tokens / 64, rounded up) at most
        const size_t tt = nexp + (np + PF_BN_SMALL - 1) / PF_BN_SMALL;
        st->cap_gu = (int)(((2 * effn + pg::BM - 1) / pg::BM) * tt), st->cap_dn = (int)(((H + pg::BM - 1) / pg::BM) * tt);
        st->t_gu = (pg::Tile *)st->alloc(st->cap_gu * sizeof(pg::Tile), &err);
        st->t_dn = (pg::Tile *)st->alloc(st->cap_dn * sizeof(pg::Tile), &err);
    }
    st->maps_cap = 64 + e->L.size() * (40 + 2 * nexp);  // (a Q6_K matrix takes four maps)
    st->maps = (CUtensorMap *)st->alloc(st->maps_cap * sizeof(CUtensorMap), &err);
    if (err != cudaSuccess) {
        delete st;
        return fail("cudaMalloc(prefill buffers)", err);
    }
    e->pf = st;
    *out = st;
    return 0;
}

// One call's work, enqueued twice: a planning pass (the dense launches' tile tables and
// every output descriptor collected on the host, weight maps built) and, after one upload
// of the tables, the pass that launches.  Both passes take the same path.
struct PfRun {
    sb_ctx *c;
    sb_engine *e;
    PfState *st;
    cudaStream_t s;
    int n, pos0;
    bool plan = true;
    std::vector<pg::Tile> tiles;  // dense launches' tiles, in launch order
    std::vector<pg::Out> outs;    // every launch's output descriptors
    std::vector<std::pair<size_t, size_t>> spans;
    size_t i_span = 0, i_out = 0;
    pg::Tile *d_tiles = nullptr;
    pg::Out *d_outs = nullptr;
    size_t launches = 0;
    // a block of hidden rows instead of the tokens' embeddings, and the rows the layers leave
    // instead of the last token's logits (the layers of one call of sb_moe_layer)
    const float *h_in = nullptr;
    float *h_out = nullptr;

    int map_index(const EngMat &m)
    {
        auto it = st->map_of.find(m.w);
        if (it != st->map_of.end()) return it->second;
        CUtensorMap h[4];
        const int nm = pg::make_wmaps(h, m.dt, m.w, (int)m.rows, (int)m.cols);
        if (nm < 1 || st->maps_n + nm > st->maps_cap) return -1;
        if (cudaMemcpy(st->maps + st->maps_n, h, nm * sizeof(CUtensorMap), cudaMemcpyHostToDevice) != cudaSuccess)
            return -1;
        const int first = (int)st->maps_n;
        st->map_of[m.w] = first;
        st->maps_n += nm;
        return first;
    }

    // a contiguous block of maps for a list of matrices (the experts of a layer), built once
    int map_block(const EngMat *ms, size_t stride, size_t count)
    {
        auto it = st->blocks.find(ms);
        if (it != st->blocks.end()) return it->second;
        if (st->maps_n + count > st->maps_cap) return -1;
        std::vector<CUtensorMap> h(count);
        for (size_t i = 0; i < count; i++) {
            const EngMat &m = ms[i * stride];
            if (pg::make_wmap(&h[i], m.dt, m.w, (int)m.rows, (int)m.cols)) return -1;
        }
        if (cudaMemcpy(st->maps + st->maps_n, h.data(), count * sizeof(CUtensorMap), cudaMemcpyHostToDevice) !=
            cudaSuccess)
            return -1;
        const int b = (int)st->maps_n;
        st->maps_n += count;
        return st->blocks[ms] = b;
    }

    const CUtensorMap *xmap(const void *x, int rows, int cols, int bn)
    {
        auto key = std::make_tuple(x, rows, cols, bn);
        auto it = st->xmaps.find(key);
        if (it != st->xmaps.end()) return &it->second;
        CUtensorMap m;
        if (pg::make_xmap(&m, x, rows, cols, bn, true)) return nullptr;
        return &(st->xmaps[key] = m);
    }

    // the index of the next output descriptor (planned: appended)
    int out(const pg::Out &o)
    {
        if (plan) {
            outs.push_back(o);
            return (int)outs.size() - 1;
        }
        return (int)i_out++;
    }

    // One dense GEMM launch: matrices ms (one dtype, cols = X's width) over X rows
    // [tok0, tok0 + ntok) (X has xrows rows), outputs os.
    int gemm(const EngMat *const *ms, const pg::Out *os, int nm, const void *x, int xrows, int tok0, int ntok)
    {
        const uint8_t dt = ms[0]->dt;
        const int cols = (int)ms[0]->cols;
        int rows_total = 0;
        for (int i = 0; i < nm; i++) {
            if (ms[i]->dt != dt || (int)ms[i]->cols != cols) return fail("prefill: a GEMM launch with mixed matrices");
            rows_total += (int)ms[i]->rows;
        }
        const int bn = pick_bn(rows_total, ntok, sb::num_sms_cached());
        if (plan) {
            const size_t t0 = tiles.size();
            for (int i = 0; i < nm; i++) {
                const int mi = map_index(*ms[i]);
                if (mi < 0) return fail("prefill: weight map of a matrix failed");
                const int oi = out(os[i]);
                for (int j = 0; j < ntok; j += bn)
                    for (int r = 0; r < (int)ms[i]->rows; r += pg::BM)
                        tiles.push_back(pg::Tile{mi, oi, r, tok0 + j, std::min(bn, ntok - j), 0, 0, 0});
            }
            spans.push_back({t0, tiles.size() - t0});
            return 0;
        }
        for (int i = 0; i < nm; i++) out(os[i]);
        const auto sp = spans[i_span++];
        const CUtensorMap *xm = xmap(x, xrows, cols, bn);
        if (!xm) return fail("prefill: X tensor map failed");
        pg::Launch a{st->maps, d_outs, d_tiles + sp.first, nullptr, cols};
        const int rc = pg::launch(dt, bn, SBK_PREC_F16, *xm, a, (int)sp.second, 1, s);
        if (rc) return fail("prefill: GEMM launch rejected (" + std::to_string(rc) + ")");
        launches++;
        return 0;
    }

    // A grouped launch over a device-written table (the experts of a MoE layer).
    int gemm_grouped(uint8_t dt, int cols, const void *x, int xrows, const pg::Tile *t, const int *count, int cap)
    {
        if (plan) return 0;
        const CUtensorMap *xm = xmap(x, xrows, cols, PF_BN_SMALL);
        if (!xm) return fail("prefill: X tensor map failed");
        pg::Launch a{st->maps, d_outs, t, count, cols};
        const int rc = pg::launch(dt, PF_BN_SMALL, SBK_PREC_F16, *xm, a, cap, 1, s);
        if (rc) return fail("prefill: grouped GEMM launch rejected (" + std::to_string(rc) + ")");
        launches++;
        return 0;
    }

    template <typename... KArgs, typename... Args>
    int ks(const char *what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args)
    {
        if (plan) return 0;
        if (sb::launch_k(kern, grid, block, smem, 1, s, args...)) return fail(std::string("prefill: launch of ") + what);
        launches++;
        return 0;
    }
    template <typename... KArgs, typename... Args>
    int k(const char *what, void (*kern)(KArgs...), dim3 grid, dim3 block, Args... args)
    {
        return ks(what, kern, grid, block, 0, args...);
    }
};

#define PF_CHECK(x)                  \
    do {                             \
        const int _rc = (x);         \
        if (_rc) return _rc;         \
    } while (0)

int pf_layers(PfRun &r)
{
    sb_engine *e = r.e;
    PfState *st = r.st;
    const int n = r.n, pos0 = r.pos0, H = (int)e->H, T = pos0 + n;
    const int cap = (int)st->cap;
    float *hc = st->h0, *ho = st->h1;  // residual stream (current / other)
    const float *yp = nullptr;         // output of the last block, still to be added
    if (r.h_in) {  // the hidden rows the caller gave
        if (!r.plan && cudaMemcpyAsync(hc, r.h_in, (size_t)n * H * 4, cudaMemcpyDeviceToDevice, r.s) != cudaSuccess)
            return fail("prefill: hidden rows copy");
    } else {
        // embedding rows of the tokens (Runtime::embed_token, runtime.rs:787-802)
        PF_CHECK(r.k("embed", sb::embed_kernel, dim3(n), dim3(256), (const uint8_t *)e->emb.w, (int)e->emb.dt,
                     (int)e->V, H, (const int *)st->tok, hc));
    }
    auto norm = [&](const float *w, float *x32) -> int {
        PF_CHECK(r.k("norm", blk::norm16_rows_kernel, dim3(n), dim3(256), (const float *)hc, yp, yp ? ho : nullptr, w,
                     st->x16, x32, H, e->eps));
        if (yp) std::swap(hc, ho);
        yp = nullptr;
        return 0;
    };
    auto to16 = [&](const float *x, __half *y, long long count) -> int {
        const long long q4 = count / 4;
        return r.k("to16", blk::to16_kernel, dim3((unsigned)std::min<long long>((q4 + 255) / 256, 4096)), dim3(256), x,
                   y, q4);
    };
    for (size_t l = 0; l < e->L.size(); l++) {
        EngLayer &L = e->L[l];
        // ---- attention
        PF_CHECK(norm(L.na, nullptr));
        if (L.mla) {
            const int qk = (int)(L.qk_nope + L.qk_rope);
            {
                const EngMat *ms[2] = {&L.q_down, &L.kv_down};
                const pg::Out os[2] = {{st->cq, (int)L.q_rank, (int)L.q_rank, 0, pg::OUT_F32},
                                       {st->c, (int)L.kv_rank, (int)L.kv_rank, 0, pg::OUT_F32}};
                PF_CHECK(r.gemm(ms, os, 2, st->x16, cap, 0, n));
            }
            PF_CHECK(r.k("latent rows", blk::mla_latent_rows_kernel, dim3(256), dim3(256), (const float *)st->c,
                         L.latent, n, (int)L.kv_rank, pos0));
            PF_CHECK(to16(st->cq, st->cq16, (long long)n * L.q_rank));
            {
                const EngMat *ms[1] = {&L.q_up};
                const pg::Out os[1] = {{st->q, (int)(L.heads * qk), (int)(L.heads * qk), 0, pg::OUT_F32}};
                PF_CHECK(r.gemm(ms, os, 1, st->cq16, cap, 0, n));
            }
            // every cached latent row re-expanded: K (f32, then roped and f16) and V (f16)
            {
                const EngMat *ms[1] = {&L.k_up};
                const pg::Out os[1] = {{st->kexp, (int)(L.kvh * qk), (int)(L.kvh * qk), 0, pg::OUT_F32}};
                PF_CHECK(r.gemm(ms, os, 1, L.latent, (int)e->ctx, 0, T));
            }
            {
                const EngMat *ms[1] = {&L.v_up};
                const pg::Out os[1] = {{st->v16, (int)(L.kvh * L.v_dim), (int)(L.kvh * L.v_dim), 0, pg::OUT_F16}};
                PF_CHECK(r.gemm(ms, os, 1, L.latent, (int)e->ctx, 0, T));
            }
            PF_CHECK(r.k("mla rope k", blk::mla_rope_rows_kernel, dim3(T), dim3(256), st->kexp, (int)L.kvh,
                         (int)L.qk_nope, (int)L.qk_rope, 0, L.theta, st->k16, L.krope, pos0));
            PF_CHECK(r.k("mla rope q", blk::mla_rope_rows_kernel, dim3(n), dim3(256), st->q, (int)L.heads,
                         (int)L.qk_nope, (int)L.qk_rope, pos0, L.theta, (uint16_t *)nullptr, (float *)nullptr, 0));
            blk::AttnPrefillArgs aa{st->q, st->k16, st->v16, st->att, n, pos0, (int)L.heads, (int)L.kvh, qk,
                                    (int)L.v_dim, (int)L.heads * qk, (int)L.kvh * qk, (int)(L.kvh * L.v_dim),
                                    (int)(L.heads * L.v_dim), 1.0f / sqrtf((float)qk)};
            if (!r.plan && blk::attn_prefill(aa, r.s)) return fail("prefill: MLA attention launch rejected");
            r.launches += r.plan ? 0 : 1;
        } else {
            const int qkv_w = (int)(L.qd + 2 * L.kvd);
            {
                const EngMat *ms[3] = {&L.q, &L.k, &L.v};
                const pg::Out os[3] = {{st->qkv, (int)L.qd, qkv_w, 0, pg::OUT_F32},
                                       {st->qkv, (int)L.kvd, qkv_w, (int)L.qd, pg::OUT_F32},
                                       {st->qkv, (int)L.kvd, qkv_w, (int)(L.qd + L.kvd), pg::OUT_F32}};
                PF_CHECK(r.gemm(ms, os, 3, st->x16, cap, 0, n));
            }
            blk::RopeRowsArgs ra{st->qkv, L.bias, L.qn, L.kn, L.kc, L.vc, pos0, (int)L.heads, (int)L.kvh, (int)L.hd,
                                 (int)e->ctx, L.theta, e->eps, L.neox, L.rf, L.rms};
            PF_CHECK(r.k("rope rows", blk::rope_kv_rows_kernel, dim3((unsigned)(L.heads + 2 * L.kvh), n),
                         dim3((unsigned)L.hd / 2), ra));
            blk::AttnPrefillArgs aa{st->qkv, L.kc, L.vc, st->att, n, pos0, (int)L.heads, (int)L.kvh, (int)L.hd,
                                    (int)L.hd, qkv_w, (int)L.kvd, (int)L.kvd, (int)L.qd, 1.0f / sqrtf((float)L.hd)};
            if (!r.plan && blk::attn_prefill(aa, r.s)) return fail("prefill: attention launch rejected");
            r.launches += r.plan ? 0 : 1;
        }
        PF_CHECK(to16(st->att, st->att16, (long long)n * L.qd));
        {
            const EngMat *ms[1] = {&L.o};
            const pg::Out os[1] = {{st->y, H, H, 0, pg::OUT_F32}};
            PF_CHECK(r.gemm(ms, os, 1, st->att16, cap, 0, n));
        }
        yp = st->y;
        // ---- FFN
        if (!L.moe) {
            PF_CHECK(norm(L.nf, nullptr));
            {
                const EngMat *ms[1] = {&L.gu2};
                const pg::Out os[1] = {{st->act16, (int)L.gu2.rows, (int)L.ffn, 0, pg::OUT_SWIGLU16}};
                PF_CHECK(r.gemm(ms, os, 1, st->x16, cap, 0, n));
            }
            if (pf_gemm_dtype(L.d.dt)) {
                const EngMat *ms[1] = {&L.d};
                const pg::Out os[1] = {{st->y, H, H, 0, pg::OUT_F32}};
                PF_CHECK(r.gemm(ms, os, 1, st->act16, cap, 0, n));
            } else {
                // a down format without the GEMM (Q6_K): the matvec kernel, 40 tokens a launch
                PF_CHECK(r.k("act f32", sb::f16_to_f32_kernel, dim3(1024), dim3(256), (const uint16_t *)st->act16,
                             st->act32, (int)(n * L.ffn)));
                for (int t0 = 0; t0 < n && !r.plan; t0 += sb::tcmv::MAXB) {
                    sbk_mv_op ops[sb::tcmv::MAXB];
                    const int m = std::min(n - t0, sb::tcmv::MAXB);
                    for (int j = 0; j < m; j++)
                        ops[j] = sbk_mv_op{L.d.w, L.d.rows, L.d.cols, st->act32 + (size_t)(t0 + j) * L.ffn,
                                           st->y + (size_t)(t0 + j) * H};
                    if (sbk_matvec_batch(L.d.dt, ops, m, 1, r.s)) return fail("prefill: down matvec batch rejected");
                    r.launches++;
                }
            }
            yp = st->y;
            continue;
        }
        // MoE FFN
        const bool f32_router = L.router.dt == SB_DTYPE_F32;
        PF_CHECK(norm(L.nf, L.sg || f32_router ? st->x32 : nullptr));
        if (f32_router) {  // the router in f32, as the reference keeps it
            PF_CHECK(r.k("router logits", blk::router_logits_f32_kernel, dim3((unsigned)((L.n_exp + 7) / 8), n),
                         dim3(256), (const float *)L.router.w, (const float *)st->x32, st->rlog, (int)L.n_exp, H));
        } else {
            const EngMat *ms[1] = {&L.router};
            const pg::Out os[1] = {{st->rlog, (int)L.n_exp, (int)L.n_exp, 0, pg::OUT_F32}};
            PF_CHECK(r.gemm(ms, os, 1, st->x16, cap, 0, n));
        }
        // (dynamic shared memory: the probabilities of one token)
        PF_CHECK(r.ks("router", sb::router_topk_kernel, dim3(n), dim3(256), L.n_exp * 4, (const float *)st->rlog,
                      (int)L.n_exp, (int)L.top_k, st->idx, st->wts));
        const int nl = (int)(L.ex_hi - L.ex_lo);
        const int mg = r.map_block(&L.ex[0], 3, nl);
        const int md = r.map_block(&L.ex[2], 3, nl);
        if (mg < 0 || md < 0) return fail("prefill: expert weight maps failed");
        const int og = r.out(pg::Out{st->actg16, (int)L.ex[0].rows, (int)L.effn, 0, pg::OUT_SWIGLU16});
        const int od = r.out(pg::Out{st->yd, H, H, 0, pg::OUT_F32});
        blk::GroupArgs ga{st->idx, n, (int)L.top_k, (int)L.n_exp, PF_BN_SMALL, (int)L.ex[0].rows, H, mg, md, og, od,
                          st->pair_slot, st->slot_tok, st->t_gu, st->t_dn, st->ntile, st->ntile + 1, st->cap_gu,
                          st->cap_dn};
        PF_CHECK(r.k("moe group", blk::moe_group_kernel, dim3(1), dim3(1024), ga));
        const int np = n * (int)L.top_k;
        PF_CHECK(r.k("moe gather", blk::moe_gather16_kernel, dim3(np), dim3(128), (const __half *)st->x16,
                     (const int *)st->slot_tok, st->xg16, np, H));
        PF_CHECK(r.gemm_grouped(L.ex[0].dt, H, st->xg16, cap * (int)L.top_k, st->t_gu, st->ntile, st->cap_gu));
        PF_CHECK(r.gemm_grouped(L.ex[2].dt, (int)L.effn, st->actg16, cap * (int)L.top_k, st->t_dn, st->ntile + 1,
                                st->cap_dn));
        if (L.sh_here) {
            const int sffn = (int)L.sh[0].rows / 2;
            {
                const EngMat *ms[1] = {&L.sh[0]};
                const pg::Out os[1] = {{st->acts16, (int)L.sh[0].rows, sffn, 0, pg::OUT_SWIGLU16}};
                PF_CHECK(r.gemm(ms, os, 1, st->x16, cap, 0, n));
            }
            {
                const EngMat *ms[1] = {&L.sh[2]};
                const pg::Out os[1] = {{st->ysh, H, H, 0, pg::OUT_F32}};
                PF_CHECK(r.gemm(ms, os, 1, st->acts16, cap, 0, n));
            }
        }
        blk::CombineArgs ca{hc, st->yd, st->pair_slot, st->wts, L.sh_here ? st->ysh : nullptr, L.sg, st->x32, ho, H,
                            (int)L.top_k};
        PF_CHECK(r.k("moe combine", blk::moe_combine_rows_kernel, dim3(n), dim3(256), ca));
        std::swap(hc, ho);
        yp = nullptr;
    }
    if (r.h_out) {  // the hidden rows the layers leave, with a pending block output added
        if (yp) return r.k("add rows", blk::add_rows_kernel, dim3(256), dim3(256), (const float *)hc, yp, r.h_out,
                           (long long)n * H);
        if (!r.plan && cudaMemcpyAsync(r.h_out, hc, (size_t)n * H * 4, cudaMemcpyDeviceToDevice, r.s) != cudaSuccess)
            return fail("prefill: hidden rows copy");
        return 0;
    }
    // the last token: hidden vector (before the output norm) and logits
    {
        const size_t last = (size_t)(n - 1) * H;
        sbk_xsrc xs{};
        xs.res = yp ? yp + last : nullptr;
        xs.norm_w = e->fnorm, xs.h_out = e->hfin, xs.eps = e->eps, xs.mode = SBK_XS_NORM;
        if (!r.plan) {
            if (!yp) {  // the residual is final already: the norm reads it as it is
                if (cudaMemcpyAsync(e->hfin, hc + last, H * 4, cudaMemcpyDeviceToDevice, r.s) != cudaSuccess)
                    return fail("prefill: hidden copy");
                xs.h_out = nullptr;
            }
            const EngMat *ms[1] = {&e->lm};
            float *ys[1] = {e->logits};
            size_t nl = 0;
            const int rc = run_mv(e, ms, ys, 1, hc + last, xs, r.s, &nl);
            if (rc) return fail("prefill: output matvec rejected (" + std::to_string(rc) + ")");
            r.launches += nl;
            if (sbk_argmax(e->logits, e->V, e->ints + 1, e->am_ws, 1, r.s)) return fail("prefill: argmax rejected");
            r.launches++;
        }
    }
    return 0;
}

// The block path over engine e for n rows at positions pos0..: a planning pass (the dense
// launches' tile tables and every output descriptor collected on the host, weight maps
// built), one upload of the tables (and of the tokens, when given), then the pass that
// launches.  Input: the tokens' embeddings, or h_in (device, n x H); output: the last token's
// logits and argmax in the engine, or h_out (device, n x H).
int pf_run(sb_ctx *c, sb_engine *e, size_t n, size_t pos0, const int32_t *tokens, const float *h_in, float *h_out,
           PfRun *out)
{
    cudaError_t err = cudaSuccess;
    PfState *st = nullptr;
    int rc = pf_state(c, e, n, &st);
    if (rc) return rc;
    PfRun &r = *out;
    r.c = c, r.e = e, r.st = st, r.s = c->stream, r.n = (int)n, r.pos0 = (int)pos0, r.h_in = h_in, r.h_out = h_out;
    if ((rc = pf_layers(r))) return rc;  // plan
    // tables up: dense tiles and output descriptors (grown as needed), then the tokens
    const size_t tb = r.tiles.size() * sizeof(pg::Tile), ob = r.outs.size() * sizeof(pg::Out);
    const size_t kb = tokens ? n * 4 : 0;
    if (r.tiles.size() > st->tiles_cap) {
        void *p = st->alloc(tb, &err);
        if (err != cudaSuccess) return fail("cudaMalloc(prefill tiles)", err);
        st->tiles = (pg::Tile *)p, st->tiles_cap = r.tiles.size();
    }
    if (r.outs.size() > st->outs_cap) {
        void *p = st->alloc(ob, &err);
        if (err != cudaSuccess) return fail("cudaMalloc(prefill outputs)", err);
        st->outs = (pg::Out *)p, st->outs_cap = r.outs.size();
    }
    if (c->ensure_host_stage(tb + ob + kb + 1024)) return -1;
    char *hs = (char *)c->host_stage;
    memcpy(hs, r.tiles.data(), tb);
    memcpy(hs + tb, r.outs.data(), ob);
    if (kb) memcpy(hs + tb + ob, tokens, kb);
    if ((tb && (err = cudaMemcpyAsync(st->tiles, hs, tb, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess) ||
        (ob && (err = cudaMemcpyAsync(st->outs, hs + tb, ob, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess) ||
        (kb && (err = cudaMemcpyAsync(st->tok, hs + tb + ob, kb, cudaMemcpyHostToDevice, c->stream)) != cudaSuccess))
        return fail("cudaMemcpyAsync(prefill tables)", err);
    r.plan = false;
    r.d_tiles = st->tiles, r.d_outs = st->outs;
    return pf_layers(r);
}

}  // namespace

extern "C" int sb_decode_prefill(sb_ctx *c, const int32_t *tokens, size_t n, size_t pos0, float *logits,
                                 int32_t *next)
{
    if (!c) return fail("null context");
    if (!tokens || !n) return fail("null argument");
    std::lock_guard<std::mutex> lk(c->mu);
    sb_engine *e = c->eng;
    if (!e || e->tp || e->pending_finish || !e->emb.w) return 0;
    if (pos0 + n > e->ctx) return fail("sb_decode_prefill: beyond the prepared context");
    for (size_t i = 0; i < n; i++)
        if (tokens[i] < 0 || (size_t)tokens[i] >= e->V) return fail("sb_decode_prefill: token id out of range");
    // what the block path takes: GEMM formats for the attention and FFN matrices, pair
    // matrices for gate / up
    for (auto &L : e->L) {
        const EngMat *need[8] = {&L.o};
        int k = 1;
        if (L.mla) need[k++] = &L.q_down, need[k++] = &L.kv_down, need[k++] = &L.q_up, need[k++] = &L.k_up,
                   need[k++] = &L.v_up;
        else need[k++] = &L.q, need[k++] = &L.k, need[k++] = &L.v;
        for (int j = 0; j < k; j++)
            if (!pf_gemm_dtype(need[j]->dt) || need[j]->cols % 256) return 0;
        if (L.mla && !blk::attn_prefill_takes((int)(L.qk_nope + L.qk_rope), (int)L.v_dim, (int)(L.heads / L.kvh)))
            return 0;
        if (!L.mla && !blk::attn_prefill_takes((int)L.hd, (int)L.hd, (int)(L.heads / L.kvh))) return 0;
        if (L.moe) {
            if (!L.ex_pairs || !(pf_gemm_dtype(L.router.dt) || L.router.dt == SB_DTYPE_F32) ||
                !pf_group_dtype(L.ex[0].dt) ||
                !pf_group_dtype(L.ex[2].dt) || L.effn % 64 || (L.sh_here && (L.sh[0].rows / 2) % 64))
                return 0;
        } else if (!L.gu2.w || !pf_gemm_dtype(L.gu2.dt) || L.ffn % 64) {
            return 0;
        }
    }
    cudaError_t err = cudaSetDevice(c->device);
    if (err != cudaSuccess) return fail("cudaSetDevice", err);
    const uint64_t t0 = now_ns();
    PfRun r;
    int rc = pf_run(c, e, n, pos0, tokens, nullptr, nullptr, &r);
    if (rc) return rc;
    const size_t tb = r.tiles.size() * sizeof(pg::Tile), ob = r.outs.size() * sizeof(pg::Out);
    char *hs;
    // the host's copy of the result: the next token and, when asked, the logits
    const size_t lb = (e->V * 4 + 255) & ~(size_t)255;
    if (c->ensure_host_stage(lb + 256)) return -1;
    hs = (char *)c->host_stage;
    if ((err = cudaMemcpyAsync(hs + lb, e->ints + 1, 4, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess ||
        (logits && (err = cudaMemcpyAsync(hs, e->logits, e->V * 4, cudaMemcpyDeviceToHost, c->stream)) != cudaSuccess))
        return fail("cudaMemcpyAsync(prefill result)", err);
    if ((err = cudaStreamSynchronize(c->stream)) != cudaSuccess) return fail("prefill", err);
    if (logits) memcpy(logits, hs, e->V * 4);
    if (next) *next = *(int32_t *)(hs + lb);
    c->stats.launches += r.launches;
    c->stats.bytes_up += tb + ob + n * 4;
    c->stats.bytes_down += 4 + (logits ? e->V * 4 : 0);
    c->stats.total_ns += now_ns() - t0;
    return 1;
}
