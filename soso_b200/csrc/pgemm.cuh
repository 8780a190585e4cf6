// pgemm.cuh -- the block-prefill GEMM on the sm_100a tensor cores, driven by a table of
// output tiles so that one launch serves several matrices that read the same input (q|k|v,
// q_down|kv_down) or the token groups of many experts (a MoE layer: every expert's rows
// times the tokens routed to it).
//
//   Y[t][yoff + r] = sum_k X[t][k] . W_m[r][k]     for the tiles (m, rows, tokens) listed
//
// Replaces the reference's block-prefill GEMMs: iq_matmul_mma / iq_gateup_mma /
// iq_down_mma (lxdde/ports/nouveau/matvec_iq.cu:731-816, :949-970; f16 mma.sync on weights
// decoded to shared memory) and the grouped expert kernels mo_gateup_grp / mo_down_grp
// (gemma_capa.cu:1174, :1223), behind GpuDispatch::matmul / expertos_bloque
// (crates/soso-llm-core/src/gpu.rs:443-475).
//
// The machinery is the dense GEMM's (prefill.cuh): tcgen05.mma kind::f16 with the D tile
// [128 weight rows x BN tokens] f32 in tensor memory, A = weight rows dequantised by eight
// warps into 128-byte-swizzled K-major shared memory, B = X (16-bit, written by an earlier
// kernel) by TMA with the 128-byte swizzle, a 3-stage ring; the raw weight block columns come
// by TMA from a warp of their own, two columns ahead of the dequantisers.
// New here: the weight formats are traits (Q4_K, and Q8_0 with 16-byte-aligned rows), the
// token tile BN is 64 or 256 (a routed expert sees ~n*top_k/n_exp tokens), every CTA finds
// its tile in a table (device-written for MoE: CTAs past the table's count leave at once),
// and the epilogue stores f32, f16 (the next GEMM's operand) or, for a matrix of gate / up
// 16-row group pairs, silu(gate) * up as f16 (swiglu_inplace, gemm.rs:210-226).
#pragma once
#include "prefill.cuh"

namespace sb {
namespace pg {

constexpr int BM = pf::BM, BK = pf::BK, NST = pf::NST, NRAW = pf::NRAW, NDQ = pf::NDQ;
// warp 0: X loads, warp 1: MMA issue, warps 2..9: dequantisers / epilogue, warp 10: raw weight loads
constexpr int RAW_WARP = 2 + NDQ, THREADS = (RAW_WARP + 1) * 32;

// One output tile: weight map `map` and output descriptor `out` of the launch's tables,
// weight rows [row0, row0 + 128), X / Y rows [tok0, tok0 + ntok) with ntok <= BN.
struct __align__(16) Tile {
    int map, out, row0, tok0, ntok, pad0, pad1, pad2;
};

enum { OUT_F32 = 0, OUT_F16 = 1, OUT_SWIGLU16 = 2 };

// Where matrix m's rows go: Y row t (a token, or a routed (token, choice) pair) at element
// yoff of a row of ldy elements.  OUT_SWIGLU16: the matrix's rows are 16-row groups of gate
// then up rows (its feature f = 16 (r / 32) + r % 16), Y gets rows / 2 features.
struct __align__(16) Out {
    void *y;
    int rows, ldy, yoff, mode;
};

struct Launch {
    const CUtensorMap *maps;  // weight maps (device memory, 64-byte aligned), by Tile::map
    const Out *outs;          // output descriptors, by Tile::out
    const Tile *tiles;        // [grid]
    const int *n_tiles;       // tiles in use (device, written by an earlier kernel), or null: all
    int cols;                 // K, the same for every matrix: a multiple of 64
};

// Weight formats: RAWB bytes of one row per raw block column (SPR stages of 64 columns:
// the unit the raw TMA ring moves), and the dequantisation of 32 weights (columns 32h.. of
// stage p of the column) into one 128-byte swizzled row of the stage tile.  Both formats
// keep a raw column at 144 bytes a row, so that at BN = 64 two CTAs fit on an SM.
// Formats held row-interleaved (a raw column is one box of 128 rows x RAWB bytes, one map).
template <class W>
struct RowRaw {
    static constexpr int NMAP = 1;
    __device__ __forceinline__ static void load_raw(uint8_t *slot, const CUtensorMap *maps, int rk, int row0, int,
                                                    uint64_t *bar, uint64_t pol)
    {
        tcmv::tma_load_2d(slot, maps, rk * (W::RAWB / 8), row0, bar, pol);
    }
    template <bool F16>
    __device__ __forceinline__ static void dq(const uint8_t *slot, int r, int, int p, int h, uint8_t *row)
    {
        W::template half16<F16>(slot + r * W::RAWB, p, h, row, r);
    }
    // the whole 64-column stage of row r
    template <bool F16>
    __device__ __forceinline__ static void dq_row(const uint8_t *slot, int r, int, int p, uint8_t *row)
    {
        W::template row16<F16>(slot + r * W::RAWB, p, row, r);
    }
};

struct FQ4K : RowRaw<FQ4K> {
    static constexpr int RAWB = 144;  // one Q4_K block (crates/sosomodel/src/layout.rs:63-64)
    static constexpr int SPR = 4;     // 64-column stages per raw column (256 columns)
    template <bool F16>
    __device__ __forceinline__ static void half16(const uint8_t *raw, int p, int h, uint8_t *row, int r)
    {
        pf::q4k_half_to_16<F16>(raw, p, h, row, r);
    }
    template <bool F16>
    __device__ __forceinline__ static void row16(const uint8_t *raw, int p, uint8_t *row, int r)
    {
        pf::q4k_row_to_16<F16>(raw, p, row, r);
    }
};

struct FQ80 : RowRaw<FQ80> {
    static constexpr int RAWB = 144;  // four .som Q8_0 blocks: f32 scale + 32 i8 (layout.rs:57-59)
    static constexpr int SPR = 2;     // 64-column stages per raw column (128 columns)
    // block 2p + h of the column: w_i = scale * q_i (dequant.rs:74-102), rounded once
    template <bool F16>
    __device__ __forceinline__ static void half16(const uint8_t *raw, int p, int h, uint8_t *row, int r)
    {
        const uint8_t *b = raw + (2 * p + h) * 36;
        const uint64_t sc2 = pf::dup2(*reinterpret_cast<const float *>(b)), nb2 = pf::dup2(-8388736.0f);
        const uint32_t *q = reinterpret_cast<const uint32_t *>(b + 4);
#pragma unroll
        for (int c = 0; c < 4; c++) {  // 8 weights -> one 16-byte chunk of the swizzled row
            // the codes' sign bits flipped: bytes q + 128, exact floats q after the bias
            const uint32_t w0 = q[2 * c] ^ 0x80808080u, w1 = q[2 * c + 1] ^ 0x80808080u;
            // scale * q, one rounding, two weights an instruction
            auto v = [&](uint32_t w, uint32_t s0, uint32_t s1) {
                return pf::pack16x2<F16>(pf::mul_f32x2(pf::codes2(w, s0, s1, nb2), sc2));
            };
            const uint4 out = make_uint4(v(w0, pf::SEL_B0, pf::SEL_B1), v(w0, pf::SEL_B2, pf::SEL_B3),
                                         v(w1, pf::SEL_B0, pf::SEL_B1), v(w1, pf::SEL_B2, pf::SEL_B3));
            const int chunk = 4 * h + c;
            *reinterpret_cast<uint4 *>(row + ((chunk ^ (r & 7)) << 4)) = out;
        }
    }
    template <bool F16>
    __device__ __forceinline__ static void row16(const uint8_t *raw, int p, uint8_t *row, int r)
    {
        half16<F16>(raw, p, 0, row, r);
        half16<F16>(raw, p, 1, row, r);
    }
};

// Q6_K rows repacked on upload into groups of 8 blocks laid out as planes -- [ql 8x128]
// [qh 8x64][sc 8x16][d 8x2] = 1680 bytes, a last group of m < 8 blocks the same way with m,
// padded to 16 bytes (SB_DTYPE_Q6_K_P) -- so a raw column here is half a block (128 columns,
// half n of block b): four boxes of 128 rows, one map each (box widths differ), landing as
// planes in the slot: ql[64n..] 64 B, qh[32n..] 32 B, the block's 16 scales, the group's d
// values (16 B).  Weight 32k + l of half n (GGML dequantize_row_q6_K, restated in
// crates/gguf2som/src/lib.rs:1639-1661): code = ((ql[64n + l + 32 (k & 1)] >> 4 (k >> 1)) &
// 15) | (((qh[32n + l] >> 2k) & 3) << 4), w = (d * sc[8n + 2k + l / 16]) * (code - 32) in
// f32 (d * sc is exact), then rounded to the operand type.
struct FQ6KP {
    static constexpr int RAWB = 128;  // bytes a row of the four planes
    static constexpr int SPR = 2;     // 64-column stages per raw column (128 columns)
    static constexpr int NMAP = 4;
    static constexpr int QL = 0, QH = 64 * BM, SC = 96 * BM, DD = 112 * BM;  // plane offsets in the slot
    __device__ __forceinline__ static void load_raw(uint8_t *slot, const CUtensorMap *maps, int rk, int row0,
                                                    int nb, uint64_t *bar, uint64_t pol)
    {
        const int b = rk >> 1, n = rk & 1, gi = b >> 3, w = b & 7, m = min(8, nb - 8 * gi), g0 = gi * 1680;
        // byte offsets / 8 (u64 columns of the row): all multiples of 16 bytes
        tcmv::tma_load_2d(slot + QL, maps + 0, (g0 + 128 * w + 64 * n) / 8, row0, bar, pol);
        tcmv::tma_load_2d(slot + QH, maps + 1, (g0 + 128 * m + 64 * w + 32 * n) / 8, row0, bar, pol);
        tcmv::tma_load_2d(slot + SC, maps + 2, (g0 + 192 * m + 16 * w) / 8, row0, bar, pol);
        tcmv::tma_load_2d(slot + DD, maps + 3, (g0 + 208 * m) / 8, row0, bar, pol);
    }
    template <bool F16>
    __device__ __forceinline__ static void dq(const uint8_t *slot, int r, int rk, int p, int h, uint8_t *row)
    {
        const int n = rk & 1, w = (rk >> 1) & 7, k = 2 * p + h;
        const uint4 *ql = reinterpret_cast<const uint4 *>(slot + QL + r * 64 + 32 * (k & 1));
        const uint4 *qh = reinterpret_cast<const uint4 *>(slot + QH + r * 32);
        const uint32_t scw = *reinterpret_cast<const uint32_t *>(slot + SC + r * 16 + 8 * n + 2 * k - ((2 * k) & 2));
        const int sh = (2 * k) & 2;  // the two scales at byte 8n + 2k: in the word at 8n + 2k - sh, bytes sh, sh+1
        const float d = __half2float(*reinterpret_cast<const __half *>(slot + DD + r * 16 + 2 * w));
        const float s0 = d * (float)(int8_t)((scw >> (8 * sh)) & 0xFFu);
        const float s1 = d * (float)(int8_t)((scw >> (8 * sh + 8)) & 0xFFu);
        const uint64_t nb2 = pf::dup2(-8388640.0f);  // -(2^23 + 32): codes 0..63 -> code - 32 exactly
        const int lsh = 4 * (k >> 1), hsh = 2 * k;
        const uint4 l0 = ql[0], l1 = ql[1], h0 = qh[0], h1 = qh[1];
        const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
        for (int c = 0; c < 4; c++) {  // 8 weights -> one 16-byte chunk of the swizzled row
            const uint64_t sc2 = pf::dup2(c < 2 ? s0 : s1);  // l < 16: scale 8n + 2k, else 8n + 2k + 1
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const uint32_t code = ((lw[2 * c + j] >> lsh) & 0x0F0F0F0Fu) | (((hw[2 * c + j] >> hsh) & 0x03030303u) << 4);
                o[2 * j] = pf::pack16x2<F16>(pf::mul_f32x2(pf::codes2(code, pf::SEL_B0, pf::SEL_B1, nb2), sc2));
                o[2 * j + 1] = pf::pack16x2<F16>(pf::mul_f32x2(pf::codes2(code, pf::SEL_B2, pf::SEL_B3, nb2), sc2));
            }
            const int chunk = 4 * h + c;
            *reinterpret_cast<uint4 *>(row + ((chunk ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
    // both 32-column chunks k = 2p, 2p + 1 of the stage: the qh bytes, the scale word and d
    // loaded once
    template <bool F16>
    __device__ __forceinline__ static void dq_row(const uint8_t *slot, int r, int rk, int p, uint8_t *row)
    {
        const int n = rk & 1, w = (rk >> 1) & 7;
        const uint4 *ql = reinterpret_cast<const uint4 *>(slot + QL + r * 64);
        const uint4 *qh = reinterpret_cast<const uint4 *>(slot + QH + r * 32);
        const uint32_t scw = *reinterpret_cast<const uint32_t *>(slot + SC + r * 16 + 8 * n + 4 * p);
        const float d = __half2float(*reinterpret_cast<const __half *>(slot + DD + r * 16 + 2 * w));
        const uint64_t nb2 = pf::dup2(-8388640.0f);
        const uint4 h0 = qh[0], h1 = qh[1];
        const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
        for (int h = 0; h < 2; h++) {  // k = 2p + h: ql bytes 32h.., scales at bytes 2h, 2h + 1 of scw
            const uint4 l0 = ql[2 * h], l1 = ql[2 * h + 1];
            const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
            const float s0 = d * (float)(int8_t)((scw >> (16 * h)) & 0xFFu);
            const float s1 = d * (float)(int8_t)((scw >> (16 * h + 8)) & 0xFFu);
            const int lsh = 4 * p, hsh = 2 * (2 * p + h);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const uint64_t sc2 = pf::dup2(c < 2 ? s0 : s1);
                uint32_t o[4];
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const uint32_t code =
                        ((lw[2 * c + j] >> lsh) & 0x0F0F0F0Fu) | (((hw[2 * c + j] >> hsh) & 0x03030303u) << 4);
                    o[2 * j] = pf::pack16x2<F16>(pf::mul_f32x2(pf::codes2(code, pf::SEL_B0, pf::SEL_B1, nb2), sc2));
                    o[2 * j + 1] = pf::pack16x2<F16>(pf::mul_f32x2(pf::codes2(code, pf::SEL_B2, pf::SEL_B3, nb2), sc2));
                }
                const int chunk = 4 * h + c;
                *reinterpret_cast<uint4 *>(row + ((chunk ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            }
        }
    }
};

template <class W, int BN>
struct Lay {
    static constexpr int X_BYTES = BN * BK * 2;
    static constexpr int W_BYTES = BM * BK * 2;
    static constexpr int RAW_BYTES = BM * W::RAWB;
    static constexpr size_t SMEM = 1024 + (size_t)NST * (X_BYTES + W_BYTES) + (size_t)NRAW * RAW_BYTES + 256;
};

template <int BN, bool F16>
__host__ __device__ constexpr uint32_t idesc()
{
    return (1u << 4) | ((F16 ? 0u : 1u) << 7) | ((F16 ? 0u : 1u) << 10) | ((uint32_t)(BN >> 3) << 17) |
           ((uint32_t)(BM >> 4) << 24);
}

template <int BN, bool F16>
__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t acc)
{
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc<BN, F16>()), "r"(acc)
        : "memory");
}

template <class W, int BN, bool F16>
__global__ void __launch_bounds__(THREADS, BN == 64 ? 2 : 1) pg_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const Launch a)
{
    using L = Lay<W, BN>;
    griddep_wait();  // the tile table and X are written by earlier kernels
    const int nt = a.n_tiles ? *a.n_tiles : (int)gridDim.x;
    if ((int)blockIdx.x >= nt) {
        griddep_launch();
        return;
    }
    const Tile t = a.tiles[blockIdx.x];
    const CUtensorMap *wmap = a.maps + t.map;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // aligned to 1024 by an offset from the shared array itself, so that the compiler keeps
    // every access derived from it in the shared window (ld.shared, not generic loads)
    uint8_t *b = smem_raw + ((1024u - (tcmv::smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t *sx = b, *sw = b + NST * L::X_BYTES, *sraw = sw + NST * L::W_BYTES;
    uint64_t *bar = reinterpret_cast<uint64_t *>(sraw + NRAW * L::RAW_BYTES);
    uint64_t *x_full = bar, *w_full = bar + NST, *st_empty = bar + 2 * NST, *raw_full = bar + 3 * NST,
             *raw_empty = bar + 3 * NST + NRAW, *acc_full = bar + 3 * NST + 2 * NRAW;
    uint32_t *tmem_addr = reinterpret_cast<uint32_t *>(acc_full + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KS = a.cols / BK;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NST; i++) {
            tcmv::mbar_init(&x_full[i], 1);
            tcmv::mbar_init(&w_full[i], NDQ / 2);  // a stage is one group's (four warps)
            tcmv::mbar_init(&st_empty[i], 1);
        }
        for (int i = 0; i < NRAW; i++) {
            tcmv::mbar_init(&raw_full[i], 1);
            tcmv::mbar_init(&raw_empty[i], NDQ);
        }
        tcmv::mbar_init(acc_full, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int i = 0; i < W::NMAP; i++) asm volatile("prefetch.tensormap [%0];" ::"l"(wmap + i) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         tcmv::smem_u32(tmem_addr)),
                     "r"(BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pf::fence_before_sync();
    __syncthreads();
    pf::fence_after_sync();
    const uint32_t tmem = *tmem_addr;
    bool failed = false;

    if (warp == 0) {
        if (lane == 0) {
            for (int ks = 0; ks < KS && !failed; ks++) {
                const int st = ks % NST;
                if (ks >= NST && !tcmv::mbar_wait(&st_empty[st], ((ks / NST) - 1) & 1, pf::WAIT)) {
                    failed = true;
                    break;
                }
                tcmv::mbar_expect_tx_arrive(&x_full[st], (unsigned)L::X_BYTES);
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
                    "{%2, %3}], [%4];" ::"r"(tcmv::smem_u32(sx + st * L::X_BYTES)),
                    "l"(&xmap), "r"(ks * BK), "r"(t.tok0), "r"(tcmv::smem_u32(&x_full[st]))
                    : "memory");
            }
            if (failed) set_dev_error(0x81u);
        }
    } else if (warp == RAW_WARP) {
        // raw weight block columns, as far ahead as the raw ring allows (not paced by the X
        // stages: a raw column comes from DRAM and feeds SPR stages)
        if (lane == 0) {
            const uint64_t pol = tcmv::l2_evict_first();
            const int NRK = (KS + W::SPR - 1) / W::SPR;
            for (int rk = 0; rk < NRK; rk++) {
                const int rs = rk % NRAW;
                if (rk >= NRAW && !tcmv::mbar_wait(&raw_empty[rs], ((rk / NRAW) - 1) & 1, pf::WAIT)) {
                    set_dev_error(0x85u);
                    break;
                }
                tcmv::mbar_expect_tx_arrive(&raw_full[rs], (unsigned)L::RAW_BYTES);
                W::load_raw(sraw + rs * L::RAW_BYTES, wmap, rk, t.row0, a.cols / 256, &raw_full[rs], pol);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            for (int ks = 0; ks < KS; ks++) {
                const int st = ks % NST;
                const unsigned par = (ks / NST) & 1;
                if (!tcmv::mbar_wait(&x_full[st], par, pf::WAIT) || !tcmv::mbar_wait(&w_full[st], par, pf::WAIT)) {
                    failed = true;
                    set_dev_error(0x82u);
                    break;
                }
                pf::fence_after_sync();
                const uint64_t ad = pf::sw128_desc(sw + st * L::W_BYTES), bd = pf::sw128_desc(sx + st * L::X_BYTES);
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++)  // K16 slices: 32 bytes along the swizzled row
                    mma<BN, F16>(tmem, ad + (uint64_t)(2 * kk), bd + (uint64_t)(2 * kk), (ks | kk) ? 1u : 0u);
                pf::mma_commit(&st_empty[st]);
            }
            pf::mma_commit(acc_full);  // completion of every MMA issued above (even after a failure)
        }
        __syncwarp();
    } else {
        // dequantisers: two groups of four warps take the even and the odd stages; thread t of
        // a group takes weight row t % 128 of its stages, the whole 64 columns (the halves share
        // their code bytes and block head).  A group releases a raw column after its last stage
        // in it (both groups have stages in every raw column but a last, partial one, whose
        // release nobody waits for).
        const int r = (threadIdx.x - 64) & (BM - 1), grp = (threadIdx.x - 64) / BM;
        for (int ks = grp; ks < KS && !failed; ks += 2) {
            const int st = ks % NST, rk = ks / W::SPR, rs = rk % NRAW, p = ks % W::SPR;
            if (p < 2 && !tcmv::mbar_wait(&raw_full[rs], (rk / NRAW) & 1, pf::WAIT)) failed = true;
            if (!failed && ks >= NST && !tcmv::mbar_wait(&st_empty[st], ((ks / NST) - 1) & 1, pf::WAIT)) failed = true;
            if (failed) {
                set_dev_error(0x83u);
                break;
            }
            W::template dq_row<F16>(sraw + rs * L::RAW_BYTES, r, rk, p, sw + st * L::W_BYTES + r * 128);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> MMA reads
            __syncwarp();
            if (lane == 0) {
                tcmv::mbar_arrive(&w_full[st]);
                if (ks + 2 >= (rk + 1) * W::SPR || ks + 2 >= KS) tcmv::mbar_arrive(&raw_empty[rs]);
            }
        }
        // epilogue: the accumulators of this warp's 32 lanes (weight rows)
        if (tcmv::mbar_wait(acc_full, 0, pf::WAIT)) {
            pf::fence_after_sync();
            const Out o = a.outs[t.out];
            const int q = warp & 3, rloc = 32 * q + lane, row = t.row0 + rloc;
            const int c0 = ((warp - 2) / 4) * (BN / 2);  // the two warps of a lane quadrant split the tokens
            for (int c = c0; c < c0 + BN / 2; c += 32) {
                float v[32];
                pf::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c, v);
                if (o.mode == OUT_SWIGLU16) {
                    // lanes 0-15: gate rows of 16 features, lanes 16-31: their up rows
                    const int f = ((t.row0 + 32 * q) >> 5) * 16 + (lane & 15);
                    __half *y = reinterpret_cast<__half *>(o.y);
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const float u = __shfl_down_sync(0xffffffffu, v[i], 16);
                        const int tok = c + i;
                        if (lane < 16 && tok < t.ntok && 2 * f < o.rows) {
                            const float g = v[i];
                            y[(size_t)(t.tok0 + tok) * o.ldy + o.yoff + f] = __float2half_rn(g / (1.0f + expf(-g)) * u);
                        }
                    }
                } else if (row < o.rows) {
                    if (o.mode == OUT_F16) {
                        __half *y = reinterpret_cast<__half *>(o.y);
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            if (c + i < t.ntok) y[(size_t)(t.tok0 + c + i) * o.ldy + o.yoff + row] = __float2half_rn(v[i]);
                    } else {
                        float *y = reinterpret_cast<float *>(o.y);
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            if (c + i < t.ntok) y[(size_t)(t.tok0 + c + i) * o.ldy + o.yoff + row] = v[i];
                    }
                }
            }
        } else {
            set_dev_error(0x84u);
        }
    }
    pf::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        pf::fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
    }
    griddep_launch();
}

// ------------------------------------------------------------------ host side

// Weight map of a matrix: [rows][row bytes / 8] u64, box = 128 rows x one raw block column.
// Q4_K rows as they are; Q8_0 rows padded to 16 bytes (SB_DTYPE_Q8_0_R).
inline int make_wmap(CUtensorMap *m, uint8_t dtype, const void *w, int rows, int cols)
{
    tcmv::EncodeTiledFn fn = tcmv::encode_fn();
    if (!fn) return -6;
    cuuint64_t rb;
    cuuint32_t bw;
    if (dtype == SB_DTYPE_Q4_K) {
        if (cols % 256) return -1;
        rb = (cuuint64_t)(cols / 256) * 144, bw = FQ4K::RAWB / 8;
    } else if (dtype == SB_DTYPE_Q8_0_R || (dtype == SB_DTYPE_Q8_0 && cols % 128 == 0)) {
        if (cols % 32 || cols < 128) return -1;
        rb = (cuuint64_t)(((size_t)cols / 32 * 36 + 15) & ~(size_t)15), bw = FQ80::RAWB / 8;
    } else {
        return -5;
    }
    if (((uintptr_t)w & 15) || rows < 1) return -2;
    cuuint64_t dims[2] = {rb / 8, (cuuint64_t)rows};
    cuuint64_t strides[1] = {rb};
    cuuint32_t box[2] = {bw, (cuuint32_t)BM};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(w), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -7;
}

// The weight maps of a matrix for the GEMM: one (row-interleaved formats), or four of the
// packed Q6_K rows (SB_DTYPE_Q6_K_P: the ql, qh, sc and d boxes of a half-block raw column,
// FQ6KP).  Returns the number of maps written to m[], or < 0.
inline int make_wmaps(CUtensorMap *m, uint8_t dtype, const void *w, int rows, int cols)
{
    if (dtype != SB_DTYPE_Q6_K_P) {
        const int rc = make_wmap(m, dtype, w, rows, cols);
        return rc ? rc : 1;
    }
    tcmv::EncodeTiledFn fn = tcmv::encode_fn();
    if (!fn) return -6;
    if (cols % 256 || cols < 256 || ((uintptr_t)w & 15) || rows < 1) return -1;
    const cuuint64_t rb = (cuuint64_t)tcmv::q6k_packed_row_bytes((size_t)cols);
    const cuuint32_t widths[4] = {64 / 8, 32 / 8, 16 / 8, 16 / 8};
    for (int i = 0; i < 4; i++) {
        cuuint64_t dims[2] = {rb / 8, (cuuint64_t)rows};
        cuuint64_t strides[1] = {rb};
        cuuint32_t box[2] = {widths[i], (cuuint32_t)BM};
        cuuint32_t es[2] = {1, 1};
        if (fn(&m[i], CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(w), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return -7;
    }
    return 4;
}

// X map: nrows x cols 16-bit operands (row-major), box = BN rows x 64 columns, 128-byte swizzle.
inline int make_xmap(CUtensorMap *m, const void *x, int nrows, int cols, int bn, bool f16)
{
    tcmv::EncodeTiledFn fn = tcmv::encode_fn();
    if (!fn) return -6;
    if (cols % BK || ((uintptr_t)x & 15) || nrows < 1) return -1;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)nrows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)bn};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                    const_cast<void *>(x), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -7;
}

template <class W, int BN, bool F16>
inline int launch_t(const CUtensorMap &xmap, const Launch &a, int grid, int pdl, cudaStream_t s)
{
    static size_t smem_rec[64];
    static std::mutex mu;
    {
        std::lock_guard<std::mutex> lk(mu);
        const int rc = tcmv::ensure_smem(pg_gemm_kernel<W, BN, F16>, Lay<W, BN>::SMEM, smem_rec);
        if (rc) return rc;
    }
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3((unsigned)grid);
    c.blockDim = dim3(THREADS);
    c.dynamicSmemBytes = Lay<W, BN>::SMEM;
    c.stream = s;
    c.attrs = at;
    c.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&c, pg_gemm_kernel<W, BN, F16>, xmap, a) == cudaSuccess ? 0 : -4;
}

// One launch of the table-driven GEMM: weight format by dtype (Q4_K or padded Q8_0), BN 64
// or 256, f16 operands (prec SBK_PREC_F16) or bf16.  grid = the table's length.
inline int launch(uint8_t dtype, int bn, int prec, const CUtensorMap &xmap, const Launch &a, int grid, int pdl,
                  cudaStream_t s)
{
    if (grid < 1 || a.cols % BK || a.cols < 256) return -1;
    const bool q4k = dtype == SB_DTYPE_Q4_K, f16 = prec == SBK_PREC_F16;
    if (dtype == SB_DTYPE_Q6_K_P) {  // (f16 operands: the block prefill's)
        if (a.cols % 256 || !f16) return -1;
        if (bn == 64) return launch_t<FQ6KP, 64, true>(xmap, a, grid, pdl, s);
        if (bn == 256) return launch_t<FQ6KP, 256, true>(xmap, a, grid, pdl, s);
        return -1;
    }
    if (!q4k && dtype != SB_DTYPE_Q8_0_R && dtype != SB_DTYPE_Q8_0) return -5;
    if (q4k && a.cols % 256) return -1;
#define PG_CASE(W, BN_, F)                                                                                             \
    if ((bn == BN_) && (f16 == F)) return launch_t<W, BN_, F>(xmap, a, grid, pdl, s)
    if (q4k) {
        PG_CASE(FQ4K, 64, true);
        PG_CASE(FQ4K, 256, true);
        PG_CASE(FQ4K, 64, false);
        PG_CASE(FQ4K, 256, false);
    } else {
        PG_CASE(FQ80, 64, true);
        PG_CASE(FQ80, 256, true);
        PG_CASE(FQ80, 64, false);
        PG_CASE(FQ80, 256, false);
    }
#undef PG_CASE
    return -1;
}

}  // namespace pg
}  // namespace sb
