// qtts_gemm.cuh -- weight-stationary tcgen05 GEMM of libqtts (sm_100a).
//
// Y[t][n] (+)= sum_k X[t][k] * W[n][k] for the batched paths (many
// utterances per decode step, or a long prefill): the projections become a
// dense contraction, so they run on the 5th-generation tensor cores.
//
//  - CTA tile: 128 weight rows (MMA M) x BN tokens (MMA N = 64, 128 or 256),
//    K in blocks of 64 (one 128-byte swizzle row of fp16), an optional K
//    split over blockIdx.z (2 to 8 ways).  The CTAs of one tile's split form
//    a thread-block cluster: each leaves its partial tile in its shared
//    memory, and after a cluster barrier CTA z sums rows [z/ks, (z+1)/ks) of
//    the tile over the cluster's partials in split order (distributed shared
//    memory) and stores them, or adds them to the residual: the sums come in
//    a fixed order, so the results do not vary from run to run.
//  - A operand (weights): the matrix is kept a second time in a tile-packed
//    layout (gemm_tile_pack_kernel): the 128 rows x 64 k of one stage are one
//    contiguous chunk, so one bulk copy (cp.async.bulk) brings a stage's
//    weights into shared memory.  Q8_0 (8192 int8 + 256 fp16 scales = 8704
//    bytes): warps 0-7 (two threads per weight row, 32 k each) dequantise it
//    there to two fp16 tiles, hi = fp16(q * d) and lo = q * d - hi (one fused
//    fp16 multiply-add), in the UMMA K-major 128B-swizzle layout,
//    fence.proxy.async, then an mbarrier arrival.  Float32 weights (32 KB):
//    the two tiles hi = fp16(w), lo = fp16(w - hi) already in that layout,
//    copied straight into the A buffers.  Both tiles are multiplied with the
//    same activations into one accumulator, so a weight enters the sum to
//    about 2^-22 of its value instead of fp16's 2^-11.
//  - B operand (activations, fp16 [T][K]): one TMA tiled load per stage
//    (cp.async.bulk.tensor.2d, 128B swizzle, no multicast); warp 8 lane 0
//    issues both copies of a stage.
//  - MMA: one thread issues tcgen05.mma.cta_group::1.kind::f16 (f16 x f16 ->
//    f32 in TMEM, M=128, N=BN, 4 x K=16 per stage, each for the hi and the lo
//    tile) and tcgen05.commit frees the stage; the accumulator (BN TMEM columns) is read back by warps 8-11 with
//    tcgen05.ld (warp w reads TMEM lanes 32*(w%4)..+31 = its weight rows).
//  - every mbarrier wait is bounded; a timeout sets the error word.
#pragma once
#include <cooperative_groups.h>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "qtts_decode.cuh"

namespace qtts {

constexpr int G_BM = 128;           // weight rows per CTA tile
constexpr int G_BK = 64;            // K per stage (128 bytes of fp16)
constexpr int G_THREADS = 384;   // Q8_0: warps 0-7 dequantise, 8 loads, 9 issues MMAs, 8-11 read TMEM back
constexpr int G_DQ = 256;        // dequantising threads: 2 per weight row
constexpr int G_A_BYTES = G_BM * G_BK * 2;  // 16 KB

// one tile-packed chunk: 128 rows x 64 k.  Q8_0: the values grouped by 8
// k, [8 groups][128 rows][8 values] (so that thread r reads group c of its
// row at a conflict-free address), then the scales [128 rows][2 fp16] of the
// two 32-blocks.  Float32: the hi tile then the lo tile, each the 16 KB
// image of the UMMA K-major 128B-swizzle layout (row r, group c of 8 k at
// byte (r / 8) * 1024 + (r % 8) * 128 + ((c ^ (r % 8)) * 16)).
__host__ __device__ constexpr int g_chunk_bytes(int wdt) {
    return wdt == WDT_Q8 ? G_BM * G_BK + G_BM * 4 : 2 * G_A_BYTES;
}
// the staging area of a Q8_0 chunk before dequantisation (float32 chunks
// land in the A tiles directly)
__host__ __device__ constexpr int g_raw_bytes(int wdt) { return wdt == WDT_Q8 ? g_chunk_bytes(wdt) : 0; }
// A tiles per stage: hi + lo (both formats: the weight enters the product to
// ~2^-22 of its value, not fp16's 2^-11)
__host__ __device__ constexpr int g_a_tiles(int) { return 2; }
// threads of a CTA: float32 tiles need no dequantisers, so their CTA is
// eight warps: warp 0 loads, warp 1 issues the MMAs, and all eight read TMEM
// back (two per lane quarter, each half of the columns) and run the
// epilogue; Q8_0 has eight dequantising warps in front, warp 8 loads, 9
// issues, 8-11 read TMEM back
__host__ __device__ constexpr int g_threads(int wdt) { return wdt == WDT_Q8 ? G_THREADS : 256; }
__host__ __device__ constexpr int g_warp0(int wdt) { return wdt == WDT_Q8 ? 8 : 0; }
// float32 tiles of up to 128 tokens run two CTAs per SM (BN TMEM columns and
// under 113 KB of shared memory each), so that one CTA's epilogue overlaps
// the other's main loop; the others run one CTA per SM
__host__ __device__ constexpr int g_ctas_per_sm(int wdt, int bn) { return wdt == WDT_F32 && bn <= 128 ? 2 : 1; }
// pipeline depth from the shared-memory budget (at most 6 stages)
__host__ __device__ constexpr int g_stage_bytes(int wdt, int bn) {
    return g_raw_bytes(wdt) + g_a_tiles(wdt) * G_A_BYTES + bn * 128;
}
__host__ __device__ constexpr int g_stage_budget(int wdt, int bn) {
    return g_ctas_per_sm(wdt, bn) == 2 ? 100 * 1024 : 220 * 1024;
}
__host__ __device__ constexpr int g_stages(int wdt, int bn) {
    return g_stage_budget(wdt, bn) / g_stage_bytes(wdt, bn) < 6 ? g_stage_budget(wdt, bn) / g_stage_bytes(wdt, bn) : 6;
}

struct GemmArgs {
    const uint8_t *w;  // tile-packed: chunk (row tile rt, k block kb) at (rt * K/64 + kb) * g_chunk_bytes
    int n_rows, K;
    int T;             // tokens
    float *out;        // out[t * ld + n]
    int ld;
    int atomic;        // add into out (the residual) instead of storing
    int ksplit;        // K splits (a cluster of ksplit CTAs per tile); K blocks per split = (K / G_BK) / ksplit
    int *err;          // error word (QTTS_E_TIMEOUT on a wait that gave up)
    __half *swiglu16;  // non-NULL: rows are gate/up pairs (2j, 2j+1) and the epilogue (or,
                       // with a K split, the cluster's reduction) writes fp16(silu(gate) * up)
                       // to swiglu16[t * ld16 + j]
    int ld16;
    // non-NULL q32: the QKV projection (rows [q 2048][k 1024][v 1024], so a
    // 128-row tile is one head), and the epilogue does what follows it per
    // token: q/k RMSNorm (q_norm / k_norm, eps) and RoPE at the token's
    // position, q to q32[t][2048], k and v appended to the paged cache
    // (pages of G_PAGE positions, [page][layer][k|v][head][G_PAGE][128], f32
    // or bf16)
    float *q32;
    const float *q_norm, *k_norm, *rope_cos, *rope_sin;
    float eps;
    const int *tok_seq, *tok_pos;
    void *kv_base;
    const int *kv_pages;
    int kv_mpps, kv_layers, kv_layer, kv_bf16;
    // non-NULL: the fp16 mirror of the pages (same page numbers), written
    // beside the cache for the tensor-core prefill attention
    __half *kv16;
};

constexpr int G_PAGE = 16;  // positions per page of the paged KV cache

// The fp16 mirror of one KV page (one layer, k or v, one kv head): its 16
// positions x 128 dims, 4 KB, laid out as the tensor cores read a tile of
// keys: [8-position group][64-dim atom][8 rows of 128 bytes, the 16-byte
// chunks of row r at chunk ^ (r % 8)] (the UMMA 128B swizzle), so that a
// page lands in shared memory by one bulk copy.
constexpr int KV16_PAGE = G_PAGE * 128 * 2;  // bytes
__host__ __device__ constexpr uint32_t kv16_off(int r, int d) {
    return ((r >> 3) * 2 + (d >> 6)) * 1024 + (r & 7) * 128 + ((((d & 63) >> 3) ^ (r & 7)) << 4) + (d & 7) * 2;
}
__host__ __device__ constexpr size_t kv16_page_index(int page, int layers, int layer, int which, int kvh) {
    return ((static_cast<size_t>(page) * layers + layer) * 2 + which) * 8 + kvh;  // 8 kv heads
}

// the QKV epilogue of token t at position pos (one warp): x[4] = this
// lane's dims 4L..4L+3 of head `head` (0-15 q, 16-23 k, 24-31 v); page: the
// KV page that holds pos (k and v heads)
__device__ __forceinline__ void qkv_token_epilogue(const GemmArgs &a, int head, int t, int pos, int page, float x[4],
                                                   int lane) {
    if (head < 24) {
        // the RoPE row first: its loads overlap the norm's reduction
        const int half = HD / 2, e0 = (4 * lane) & (half - 1);
        const float4 cs = *reinterpret_cast<const float4 *>(a.rope_cos + static_cast<size_t>(pos) * half + e0);
        const float4 sn = *reinterpret_cast<const float4 *>(a.rope_sin + static_cast<size_t>(pos) * half + e0);
        const float *nw = head < 16 ? a.q_norm : a.k_norm;
        const float4 g = *reinterpret_cast<const float4 *>(nw + 4 * lane);
        float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = 1.0f / sqrtf(ss / static_cast<float>(HD) + a.eps);
        x[0] = g.x * (x[0] * inv);
        x[1] = g.y * (x[1] * inv);
        x[2] = g.z * (x[2] * inv);
        x[3] = g.w * (x[3] * inv);
        const float cv[4] = {cs.x, cs.y, cs.z, cs.w}, sv[4] = {sn.x, sn.y, sn.z, sn.w};
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float partner = __shfl_xor_sync(0xffffffffu, x[j], 16);
            o[j] = lane < 16 ? x[j] * cv[j] - partner * sv[j] : x[j] * cv[j] + partner * sv[j];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = o[j];
    }
    if (head < 16) {
        *reinterpret_cast<float4 *>(a.q32 + static_cast<size_t>(t) * QDIM + head * HD + 4 * lane) =
            make_float4(x[0], x[1], x[2], x[3]);
        return;
    }
    const int which = head < 24 ? 0 : 1, kvh = head < 24 ? head - 16 : head - 24;
    const size_t e = ((((static_cast<size_t>(page) * a.kv_layers + a.kv_layer) * 2 + which) * HKV + kvh) * G_PAGE +
                      pos % G_PAGE) * HD + 4 * lane;
    if (a.kv_bf16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(x[0], x[1]), hi = __floats2bfloat162_rn(x[2], x[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t *>(&lo);
        u.y = *reinterpret_cast<uint32_t *>(&hi);
        *reinterpret_cast<uint2 *>(static_cast<__nv_bfloat16 *>(a.kv_base) + e) = u;
    } else {
        *reinterpret_cast<float4 *>(static_cast<float *>(a.kv_base) + e) = make_float4(x[0], x[1], x[2], x[3]);
    }
    if (a.kv16) {
        const __half2 lo = __floats2half2_rn(x[0], x[1]), hi = __floats2half2_rn(x[2], x[3]);
        uint2 u;
        u.x = *reinterpret_cast<const uint32_t *>(&lo);
        u.y = *reinterpret_cast<const uint32_t *>(&hi);
        uint8_t *pg = reinterpret_cast<uint8_t *>(a.kv16) +
                      kv16_page_index(page, a.kv_layers, a.kv_layer, which, kvh) * KV16_PAGE;
        *reinterpret_cast<uint2 *>(pg + kv16_off(pos % G_PAGE, 4 * lane)) = u;
    }
}

template <int WDT, int BN>
struct __align__(1024) GemmSmem {
    static constexpr int S = g_stages(WDT, BN);
    // the split-K partial tile [BN][128] f32 reuses the stage buffers
    uint8_t a[S][g_a_tiles(WDT)][G_A_BYTES];  // 1024-aligned: swizzle atoms
    uint8_t b[S][BN * 128];
    uint8_t raw[S][g_raw_bytes(WDT) > 0 ? g_raw_bytes(WDT) : 16];  // a Q8_0 stage's packed weights
    uint64_t full_raw[S];             // bulk copy tx bytes (float32: the A tiles themselves)
    uint64_t full_a[S];               // 256 dequantiser arrivals (Q8_0)
    uint64_t full_b[S];               // TMA tx bytes
    uint64_t empty[S];                // tcgen05.commit
    uint64_t accum;                   // last MMA done
    uint32_t tmem_base;
    static_assert(S * (g_a_tiles(WDT) * G_A_BYTES + BN * 128) >= G_BM * BN * 4,
                  "the split-K partial tile must fit in the stage buffers");
    static_assert(S >= 2, "at least two pipeline stages");
};

// row-packed matrix (Q8_0: [K int8][K/32 fp16] per row; f32 rows) -> the
// tile-packed chunks; rows beyond n_rows are zero.  One thread per (row of
// the padded tile grid, k block, group of 8).
__global__ void gemm_tile_pack_kernel(const uint8_t *src, int wdt, int n_rows, int K, uint8_t *dst) {
    const int KB = K / G_BK;
    const int rows_p = (n_rows + G_BM - 1) / G_BM * G_BM;
    const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<long long>(rows_p) * KB * 8) return;
    const int c = static_cast<int>(t & 7);
    const long long rk = t >> 3;
    const int kb = static_cast<int>(rk % KB);
    const int n = static_cast<int>(rk / KB);
    const int rt = n / G_BM, r = n % G_BM;
    uint8_t *chunk = dst + (static_cast<size_t>(rt) * KB + kb) * g_chunk_bytes(wdt);
    const int k = kb * G_BK + 8 * c;
    if (wdt == WDT_Q8) {
        const int rb = K + K / 16;
        uint2 q = make_uint2(0u, 0u);
        if (n < n_rows) q = *reinterpret_cast<const uint2 *>(src + static_cast<size_t>(n) * rb + k);
        *reinterpret_cast<uint2 *>(chunk + (c * G_BM + r) * 8) = q;
        if (c < 2) {
            uint16_t d = 0;
            if (n < n_rows) d = reinterpret_cast<const uint16_t *>(src + static_cast<size_t>(n) * rb + K)[kb * 2 + c];
            reinterpret_cast<uint16_t *>(chunk + G_BM * G_BK)[r * 2 + c] = d;
        }
    } else {
        float w[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (n < n_rows) {
            const float *row = reinterpret_cast<const float *>(src + static_cast<size_t>(n) * K * 4);
            const float4 a = *reinterpret_cast<const float4 *>(row + k);
            const float4 b = *reinterpret_cast<const float4 *>(row + k + 4);
            w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w, w[4] = b.x, w[5] = b.y, w[6] = b.z, w[7] = b.w;
        }
        __half hi[8], lo[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            hi[j] = __float2half_rn(w[j]);
            lo[j] = __float2half_rn(w[j] - __half2float(hi[j]));  // the difference is exact in float32
        }
        const int off = (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4);
        *reinterpret_cast<uint4 *>(chunk + off) = *reinterpret_cast<const uint4 *>(hi);
        *reinterpret_cast<uint4 *>(chunk + G_A_BYTES + off) = *reinterpret_cast<const uint4 *>(lo);
    }
}

// ------------------------------------------------------------------ tcgen05 helpers

__device__ __forceinline__ uint64_t umma_desc_sw128(const void *smem) {
    // K-major, 128B swizzle: LBO 16 B (encoded 1), SBO 1024 B (8 rows x 128 B),
    // version 1 (sm100), layout type 2 (SWIZZLE_128B), base offset 0
    const uint64_t addr = (smem_u32(smem) >> 4) & 0x3FFFull;
    return addr | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
    // c f32 (bit 4), a/b f16 (0), K-major both, N>>3 at bit 17, M>>4 at bit 24
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ __half2 u32_as_half2(uint32_t u) {
    __half2 h;
    *reinterpret_cast<uint32_t *>(&h) = u;
    return h;
}
__device__ __forceinline__ void gemm_fail(int *err) {
    if (err) atomicCAS(err, 0, ERR_TIMEOUT);
}

// ------------------------------------------------------------------ kernel

template <int WDT, int BN>
__global__ void __launch_bounds__(g_threads(WDT), g_ctas_per_sm(WDT, BN))
    gemm_kernel(const GemmArgs args, const __grid_constant__ CUtensorMap xmap) {
    using Smem = GemmSmem<WDT, BN>;
    constexpr int S = Smem::S;
    constexpr int NT = g_threads(WDT), W0 = g_warp0(WDT);  // W0: loader, W0 + 1: MMA, W0..: epilogue
    constexpr int EW = NT / 32 - W0;                      // epilogue warps: 4 or 8
    constexpr int ECOLS = BN / (EW / 4);                  // TMEM columns per epilogue warp
    static_assert(EW % 4 == 0 && ECOLS % 32 == 0, "whole lane quarters and 32-column loads");
    constexpr uint32_t CHUNK = g_chunk_bytes(WDT);
    extern __shared__ __align__(1024) uint8_t gsmem_raw[];
    // the dynamic window is aligned up to 1024 bytes (the swizzle atom)
    Smem *sm = reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(gsmem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row0 = blockIdx.x * G_BM, tok0 = blockIdx.y * BN;
    const int kb_total = args.K / G_BK, kb_n = kb_total / args.ksplit, kb0 = blockIdx.z * kb_n;
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&sm->full_raw[s], 1);
            mbar_init(&sm->full_a[s], G_DQ);
            mbar_init(&sm->full_b[s], 1);
            mbar_init(&sm->empty[s], 1);
        }
        mbar_init(&sm->accum, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == W0 + 1) {  // TMEM: BN f32 columns for the 128 x BN accumulator
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm->tmem_base)),
                     "n"(BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    pdl_trigger();
    const uint32_t tmem = sm->tmem_base;
    // every copy issued is waited for before the CTA exits (also on a
    // timeout), so no bulk copy lands in shared memory of a later CTA
    int issued = 0;

    if (warp < 8 && WDT == WDT_Q8) {
        // ---- dequantisers (Q8_0): two threads per weight row of the tile,
        // 4 of the 8 groups of 8 k each
        const int r = tid & (G_BM - 1), c0 = (tid >> 7) * 4;
        for (int i = 0; i < kb_n; ++i) {
            const int s = i % S;
            if (!mbar_wait(&sm->full_raw[s], (i / S) & 1, nullptr)) {
                gemm_fail(args.err);
                break;
            }
            const uint8_t *raw = sm->raw[s];
            uint8_t *dst = sm->a[s][0] + (r >> 3) * 1024 + (r & 7) * 128;
            uint8_t *dst_lo = sm->a[s][1] + (r >> 3) * 1024 + (r & 7) * 128;
            __half2 d2lo = __float2half2_rn(0.f), d2hi = d2lo;  // the two blocks' scales, broadcast
            if (WDT == WDT_Q8) {
                const __half2 dd = *reinterpret_cast<const __half2 *>(raw + G_BM * G_BK + r * 4);
                d2lo = __low2half2(dd);
                d2hi = __high2half2(dd);
            }
#pragma unroll
            for (int c = c0; c < c0 + 4; ++c) {  // 4 groups of 8 k
                // q + 128 in the mantissa of fp16 1024 (exact), minus 1152:
                // q exactly; hi = fp16(q * d) (the exact product rounded
                // once), lo = q * d - hi by one fused fp16 multiply-add
                __half2 h[4], lo[4];
                const uint2 q = *reinterpret_cast<const uint2 *>(raw + (c * G_BM + r) * 8);
                const uint32_t ux = q.x ^ 0x80808080u, uy = q.y ^ 0x80808080u;
                const __half2 bias = __float2half2_rn(1152.f);
                const __half2 d2 = c < 4 ? d2lo : d2hi;
                const __half2 qv[4] = {__hsub2(u32_as_half2(__byte_perm(ux, 0x64646464u, 0x5140)), bias),
                                       __hsub2(u32_as_half2(__byte_perm(ux, 0x64646464u, 0x7362)), bias),
                                       __hsub2(u32_as_half2(__byte_perm(uy, 0x64646464u, 0x5140)), bias),
                                       __hsub2(u32_as_half2(__byte_perm(uy, 0x64646464u, 0x7362)), bias)};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    h[e] = __hmul2(qv[e], d2);
                    lo[e] = __hfma2(qv[e], d2, __hneg2(h[e]));
                }
                *reinterpret_cast<uint4 *>(dst + ((c ^ (r & 7)) << 4)) = *reinterpret_cast<uint4 *>(h);
                *reinterpret_cast<uint4 *>(dst_lo + ((c ^ (r & 7)) << 4)) = *reinterpret_cast<uint4 *>(lo);
            }
            // the tensor core reads shared memory through the async proxy
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(&sm->full_a[s]);
        }
    } else if (warp == W0) {
        // ---- producer: the weight chunk (bulk copy) and the activations (TMA)
        if (lane == 0) {
            const uint8_t *wt = args.w + (static_cast<size_t>(blockIdx.x) * kb_total + kb0) * CHUNK;
            // the weights of the first stages do not depend on the previous
            // kernel: they are on their way before its completion is awaited
            const int pre = kb_n < S ? kb_n : S;
            for (int i = 0; i < pre; ++i) {
                mbar_arrive_tx(&sm->full_raw[i], CHUNK);
                bulk_g2s(WDT == WDT_Q8 ? sm->raw[i] : sm->a[i][0], wt + static_cast<size_t>(i) * CHUNK, CHUNK,
                         &sm->full_raw[i]);
            }
            pdl_wait();
            for (int i = 0; i < kb_n; ++i) {
                const int s = i % S;
                if (i >= S) {
                    if (!mbar_wait(&sm->empty[s], ((i / S) - 1) & 1, nullptr)) {
                        gemm_fail(args.err);
                        break;
                    }
                    mbar_arrive_tx(&sm->full_raw[s], CHUNK);
                    bulk_g2s(WDT == WDT_Q8 ? sm->raw[s] : sm->a[s][0], wt + static_cast<size_t>(i) * CHUNK, CHUNK,
                             &sm->full_raw[s]);
                }
                mbar_arrive_tx(&sm->full_b[s], BN * 128);
                tma_load_2d(sm->b[s], &xmap, (kb0 + i) * G_BK, tok0, &sm->full_b[s]);
                issued = i + 1;  // (a break happens at i >= S: every stage before it has both copies)
            }
        }
    } else if (warp == W0 + 1) {
        // ---- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_f16(G_BM, BN);
            for (int i = 0; i < kb_n; ++i) {
                const int s = i % S;
                const uint32_t par = (i / S) & 1;
                // Q8_0: the dequantisers' arrivals; float32: the copy itself
                uint64_t *ready = WDT == WDT_Q8 ? &sm->full_a[s] : &sm->full_raw[s];
                if (!mbar_wait(ready, par, nullptr) || !mbar_wait(&sm->full_b[s], par, nullptr)) {
                    gemm_fail(args.err);
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint64_t da = umma_desc_sw128(sm->a[s][0]), db = umma_desc_sw128(sm->b[s]);
#pragma unroll
                for (int k = 0; k < G_BK / 16; ++k) {  // +32 bytes (2 in 16-byte units) per K=16
                    umma_f16(tmem, da + 2 * k, db + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
                    // the lo tile, 16 KB (1024 16-byte units) further
                    umma_f16(tmem, da + 1024 + 2 * k, db + 2 * k, idesc, 1u);
                }
                umma_commit(&sm->empty[s]);
            }
            umma_commit(&sm->accum);
        }
    }
    // ---- epilogue: warps W0.., TMEM lane quarter = warp % 4, columns
    // [ECOLS ch, ECOLS (ch + 1)) with ch = (warp - W0) / 4
    if (warp >= W0) {
        pdl_wait();  // out may be written by the previous kernels
        const bool good = mbar_wait(&sm->accum, 0, nullptr);
        if (!good) gemm_fail(args.err);
        __syncwarp();  // tcgen05.ld is warp-wide: lane 0 of the loader and MMA warps had other work
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int q = warp & 3, ch = (warp - W0) >> 2;
        const int n = row0 + 32 * q + lane;
#pragma unroll 1
        for (int c = ECOLS * ch; c < ECOLS * (ch + 1); c += 32) {
            float v[32];
            tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + c, v);
            if (args.swiglu16 && args.ksplit == 1) {
                // the up row of a pair is the next lane: SiLU(gate) * up, as
                // the separate SwiGLU kernel computes it.  Of two columns, the
                // even lane finishes the first and the odd lane the second
                // (each sends the partner the value it lacks)
                const bool odd = lane & 1;
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    const float recv = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[j + 1], 1);
                    const float g = odd ? recv : v[j], up = odd ? v[j + 1] : recv;
                    const int t = tok0 + c + j + (odd ? 1 : 0);
                    if (good && (n & ~1) < args.n_rows && t < args.T) {
                        const float sl = g / (1.0f + expf(-g));
                        args.swiglu16[static_cast<size_t>(t) * args.ld16 + (n >> 1)] = __float2half_rn(sl * up);
                    }
                }
                continue;
            }
            if (args.ksplit > 1 || args.q32) {
                // the partial tile, [BN tokens][128 rows], over the stage
                // buffers (every copy has landed and every MMA read them)
                float *part = reinterpret_cast<float *>(sm);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 32; ++j) part[(c + j) * G_BM + 32 * q + lane] = v[j];
                continue;
            }
            if (good && n < args.n_rows) {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int t = tok0 + c + j;
                    if (t < args.T) {
                        float *o = args.out + static_cast<size_t>(t) * args.ld + n;
                        if (args.atomic)
                            atomicAdd(o, v[j]);
                        else
                            *o = v[j];
                    }
                }
            }
        }
    }
    if (args.q32) {
        // the QKV epilogue: the tile's (partial) sums [BN][128] are in shared
        // memory (of every CTA of the cluster with a K split); CTA z takes
        // tokens [z BN/ks, (z+1) BN/ks), a warp a token, sums its 128 rows
        // over the ranks in order and finishes the head
        namespace cg = cooperative_groups;
        const int ks = args.ksplit;
        int z = 0;
        if (ks > 1) {
            cg::cluster_group cl = cg::this_cluster();
            cl.sync();
            z = static_cast<int>(cl.block_rank());
        } else {
            __syncthreads();
        }
        pdl_wait();  // the pages and q32 may be read by the previous kernels
        const float *part = reinterpret_cast<const float *>(sm);
        const int per = BN / ks, head = row0 / G_BM, nw = NT / 32;
        // a warp takes tokens i = warp + nw m; their positions and pages are
        // fetched 32 at a time (lane j: the round's j-th token), then passed
        // around by shuffles
        for (int i0 = warp; i0 < per; i0 += 32 * nw) {
            int my_pos = 0, my_page = 0;
            {
                const int ij = i0 + nw * lane, tj = tok0 + z * per + ij;
                if (ij < per && tj < args.T) {
                    my_pos = args.tok_pos[tj];
                    if (head >= 16) my_page = args.kv_pages[args.tok_seq[tj] * args.kv_mpps + my_pos / G_PAGE];
                }
            }
            for (int m = 0; m < 32; ++m) {
                const int i = i0 + nw * m;
                if (i >= per) break;  // uniform over the warp
                const int col = z * per + i, t = tok0 + col;
                const int pos = __shfl_sync(0xffffffffu, my_pos, m), page = __shfl_sync(0xffffffffu, my_page, m);
                if (t >= args.T) continue;
                float x[4] = {0.f, 0.f, 0.f, 0.f};
                for (int r = 0; r < ks; ++r) {
                    const float *src = part + col * G_BM + 4 * lane;
                    if (ks > 1) src = cg::this_cluster().map_shared_rank(src, static_cast<unsigned>(r));
                    const float4 v = *reinterpret_cast<const float4 *>(src);
                    x[0] += v.x;
                    x[1] += v.y;
                    x[2] += v.z;
                    x[3] += v.w;
                }
                qkv_token_epilogue(args, head, t, pos, page, x, lane);
            }
        }
        if (ks > 1) cg::this_cluster().sync();
    } else if (args.ksplit > 1) {
        // fixed-order split-K: the cluster's partials meet, CTA z sums its
        // rows of the tile over ranks 0..ks-1 in order; a second barrier
        // keeps every CTA's shared memory alive until the others have read it
        namespace cg = cooperative_groups;
        cg::cluster_group cl = cg::this_cluster();
        cl.sync();
        pdl_wait();  // out may be written by the previous kernels
        const int ks = args.ksplit, z = static_cast<int>(cl.block_rank());
        const int rows_z = G_BM / ks, rz0 = z * rows_z;
        const float *part = reinterpret_cast<const float *>(sm);
        if (args.swiglu16) {
            // gate/up pairs (rows 2j, 2j+1; a chunk of rows_z >= 16 rows
            // holds whole pairs): fp16(silu(gate) * up) as the unsplit epilogue
            const int pz = rows_z / 2;
            for (int idx = tid; idx < pz * BN; idx += NT) {
                const int rr = rz0 + 2 * (idx % pz), col = idx / pz;
                float g = 0.f, u = 0.f;
                for (int r = 0; r < ks; ++r) {
                    const float *pr = cl.map_shared_rank(part + col * G_BM + rr, static_cast<unsigned>(r));
                    g += pr[0];
                    u += pr[1];
                }
                const int n = row0 + rr, t = tok0 + col;
                if (n < args.n_rows && t < args.T) {
                    const float sl = g / (1.0f + expf(-g));
                    args.swiglu16[static_cast<size_t>(t) * args.ld16 + (n >> 1)] = __float2half_rn(sl * u);
                }
            }
        } else {
            for (int idx = tid; idx < rows_z * BN; idx += NT) {
                const int rr = rz0 + idx % rows_z, col = idx / rows_z;
                float sum = 0.f;
                for (int r = 0; r < ks; ++r)
                    sum += *cl.map_shared_rank(part + col * G_BM + rr, static_cast<unsigned>(r));
                const int n = row0 + rr, t = tok0 + col;
                if (n < args.n_rows && t < args.T) {
                    float *o = args.out + static_cast<size_t>(t) * args.ld + n;
                    *o = args.atomic ? *o + sum : sum;
                }
            }
        }
        cl.sync();
    }
    if (warp == W0 && lane == 0) {
        // drain: wait (bounded) for the copies of the last S issued stages
        for (int i = issued > S ? issued - S : 0; i < issued; ++i) {
            const int s = i % S;
            if (!mbar_wait(&sm->full_raw[s], (i / S) & 1, nullptr) || !mbar_wait(&sm->full_b[s], (i / S) & 1, nullptr)) {
                gemm_fail(args.err);
                break;
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == W0 + 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(BN) : "memory");
    }
}

// f32 rows -> fp16 rows (the activations of the tensor-core path)
__global__ void to_half_kernel(const float *x, __half *y, long long n) {
    long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i + 3 < n) {
        const float4 v = *reinterpret_cast<const float4 *>(x + i);
        *reinterpret_cast<__half2 *>(y + i) = __floats2half2_rn(v.x, v.y);
        *reinterpret_cast<__half2 *>(y + i + 2) = __floats2half2_rn(v.z, v.w);
    } else {
        for (; i < n; ++i) y[i] = __float2half_rn(x[i]);
    }
}

}  // namespace qtts
