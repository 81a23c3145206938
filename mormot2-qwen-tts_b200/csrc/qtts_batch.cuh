// qtts_batch.cuh -- the batched forward of libqtts (sm_100a): many sequences
// (utterances) through one stack per call, the projections on the tcgen05
// GEMM (qtts_gemm.cuh, whose epilogues also do q/k-norm + RoPE + the append
// into the paged KV cache after the QKV projection, and SwiGLU after gate/up),
// the rest here: RMSNorm to fp16, causal GQA attention over the pages.
//
// Paged KV cache: pages of 16 positions; a page holds, for every layer, K and
// V of the 8 KV heads: [page][layer][k|v][head][16][128], in float32 or bf16.
// Each sequence has a page table (page of position p = table[p / 16]).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "qtts_decode.cuh"
#include "qtts_gemm.cuh"

namespace qtts {

constexpr int PAGE = G_PAGE;  // positions per page (the QKV GEMM's epilogue appends to the pages too)
constexpr int AQB = 16;    // query rows per attention item (prefill)
constexpr int AKT = 16;    // keys per attention tile
constexpr int ATHREADS = 256;

template <class KVT>
struct KVPool {
    KVT *base;
    const int *pages;  // [max_seqs][mpps]
    int mpps;          // max pages per sequence
    int layers;
};

template <class KVT>
__device__ __forceinline__ KVT *kv_at(const KVPool<KVT> &p, int layer, int seq, int pos, int which, int head) {
    const int page = p.pages[seq * p.mpps + pos / PAGE];
    return p.base + ((((static_cast<size_t>(page) * p.layers + layer) * 2 + which) * HKV + head) * PAGE + pos % PAGE) * HD;
}
__device__ __forceinline__ void store4(float *d, float4 v) { *reinterpret_cast<float4 *>(d) = v; }
__device__ __forceinline__ void store4(__nv_bfloat16 *d, float4 v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t *>(&a);
    u.y = *reinterpret_cast<uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(d) = u;
}
__device__ __forceinline__ float4 load4(const float *s) { return *reinterpret_cast<const float4 *>(s); }
__device__ __forceinline__ float4 load4(const __nv_bfloat16 *s) {
    const uint2 u = *reinterpret_cast<const uint2 *>(s);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

// One warp per row: out16[o] = fp16(rmsnorm(x[idx[o]]) * w); optionally the
// float32 normed row too (the normed state returned as `hidden`).
__global__ void rmsnorm_f16_kernel(const float *x, const int *idx, int rows, const float *w, float eps, __half *out16,
                                   float *out32) {
    pdl_trigger();
    const int o = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    // the norm weights do not depend on the previous kernel: loaded before
    // waiting for it
    float4 gw[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) gw[i] = load4(w + 4 * (lane + 32 * i));
    pdl_wait();
    if (o >= rows) return;
    const float *r = x + static_cast<size_t>(idx ? idx[o] : o) * H;
    float4 v[8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        v[i] = load4(r + 4 * (lane + 32 * i));
        ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(H) + eps);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = 4 * (lane + 32 * i);
        const float4 g = gw[i];
        const float4 y = make_float4(g.x * (v[i].x * inv), g.y * (v[i].y * inv), g.z * (v[i].z * inv), g.w * (v[i].w * inv));
        *reinterpret_cast<__half2 *>(out16 + static_cast<size_t>(o) * H + e) = __floats2half2_rn(y.x, y.y);
        *reinterpret_cast<__half2 *>(out16 + static_cast<size_t>(o) * H + e + 2) = __floats2half2_rn(y.z, y.w);
        if (out32) store4(out32 + static_cast<size_t>(o) * H + e, y);
    }
}

// One attention work item: the new rows [qa, qb) of one sequence (token t0
// is its first new row, at position L0) against keys [ka, kb) of kv head h.
struct AttnItem {
    int t0, L0, qa, qb, h, ka, kb, seq, part;  // part < 0: write the normalised output
};

// Causal GQA attention of one prefill item (several new rows of a
// sequence, all of its keys); query heads 2h and 2h+1 share kv head h.
// Warps are spread over the (row, q head) combos and, when there are fewer
// combos than warps, over the keys of each tile; their online-softmax
// states are merged in shared memory.
template <class KVT>
__global__ void __launch_bounds__(ATHREADS) attn_kernel(const AttnItem *items, const float *q32, KVPool<KVT> pool,
                                                        int layer, __half *attn16) {
    __shared__ __align__(16) float qs[AQB][2][HD];
    __shared__ __align__(16) float ks[AKT][HD];
    __shared__ __align__(16) float vs[AKT][HD];
    __shared__ __align__(16) float ws[8][HD + 4];
    pdl_trigger();
    pdl_wait();
    const AttnItem it = items[blockIdx.x];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int R = it.qb - it.qa, nc = 2 * R;
    for (int i = tid; i < R * 2 * (HD / 4); i += ATHREADS) {
        const int j = i / (2 * (HD / 4)), rem = i - j * 2 * (HD / 4), q = rem / (HD / 4), d4 = rem - q * (HD / 4);
        store4(&qs[j][q][4 * d4],
               load4(q32 + static_cast<size_t>(it.t0 + it.qa + j) * QDIM + (2 * it.h + q) * HD + 4 * d4));
    }
    // warp layout: npw warps per combo (nc <= 8), or combos w, w+8, .. per warp
    const int npw = nc <= 8 ? 8 / nc : 1;
    const int ncw = nc <= 8 ? 1 : (nc + 7) / 8;  // combos per warp
    const int kend = min(it.kb, it.L0 + it.qb);  // keys beyond the last row are masked anyway
    float m[4], l[4], o[4][4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        m[c] = -INFINITY;
        l[c] = 0.f;
        o[c][0] = o[c][1] = o[c][2] = o[c][3] = 0.f;
    }
    const float scale = 1.0f / sqrtf(static_cast<float>(HD));
    for (int kt = it.ka; kt < kend; kt += AKT) {
        const int nt = min(AKT, kend - kt);
        __syncthreads();
        for (int i = tid; i < nt * (HD / 4); i += ATHREADS) {
            const int p = i / (HD / 4), d4 = i - p * (HD / 4);
            store4(&ks[p][4 * d4], load4(kv_at(pool, layer, it.seq, kt + p, 0, it.h) + 4 * d4));
            store4(&vs[p][4 * d4], load4(kv_at(pool, layer, it.seq, kt + p, 1, it.h) + 4 * d4));
        }
        __syncthreads();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            if (c >= ncw) break;
            const int combo = nc <= 8 ? warp / npw : warp + 8 * c;
            const int sub = nc <= 8 ? warp - combo * npw : 0;
            if (combo >= nc) break;
            const int j = combo >> 1, q = combo & 1;
            const int qpos = it.L0 + it.qa + j;
            const float4 qv = load4(&qs[j][q][4 * lane]);
            for (int p = sub; p < nt; p += npw) {
                if (kt + p > qpos) break;  // causal
                const float4 kv4 = load4(&ks[p][4 * lane]);
                float d = qv.x * kv4.x;
                d = fmaf(qv.y, kv4.y, d);
                d = fmaf(qv.z, kv4.z, d);
                d = fmaf(qv.w, kv4.w, d);
                d = warp_sum(d) * scale;
                const float mn = fmaxf(m[c], d);
                const float corr = expf(m[c] - mn), e = expf(d - mn);
                l[c] = l[c] * corr + e;
                const float4 vv = load4(&vs[p][4 * lane]);
                o[c][0] = fmaf(e, vv.x, o[c][0] * corr);
                o[c][1] = fmaf(e, vv.y, o[c][1] * corr);
                o[c][2] = fmaf(e, vv.z, o[c][2] * corr);
                o[c][3] = fmaf(e, vv.w, o[c][3] * corr);
                m[c] = mn;
            }
        }
    }
    // results: merge the npw warps of a combo (nc <= 8), then write
    for (int c = 0; c < ncw; ++c) {
        int combo = nc <= 8 ? warp / npw : warp + 8 * c;
        float M = m[c], L = l[c];
        float4 acc = make_float4(o[c][0], o[c][1], o[c][2], o[c][3]);
        bool writer = combo < nc;
        if (nc <= 8) {
            __syncthreads();
            if (combo < nc) {
                store4(&ws[warp][4 * lane], acc);
                if (lane == 0) {
                    ws[warp][HD] = M;
                    ws[warp][HD + 1] = L;
                }
            }
            __syncthreads();
            writer = combo < nc && warp == combo * npw;
            if (writer) {
                M = -INFINITY;
                for (int s = 0; s < npw; ++s) M = fmaxf(M, ws[combo * npw + s][HD]);
                L = 0.f;
                acc = make_float4(0.f, 0.f, 0.f, 0.f);
                if (M != -INFINITY) {
                    for (int s = 0; s < npw; ++s) {
                        const float ms = ws[combo * npw + s][HD];
                        const float e = ms == -INFINITY ? 0.f : expf(ms - M);
                        L = fmaf(ws[combo * npw + s][HD + 1], e, L);
                        const float4 v = load4(&ws[combo * npw + s][4 * lane]);
                        acc.x = fmaf(v.x, e, acc.x);
                        acc.y = fmaf(v.y, e, acc.y);
                        acc.z = fmaf(v.z, e, acc.z);
                        acc.w = fmaf(v.w, e, acc.w);
                    }
                }
            }
        }
        if (!writer) continue;
        const int j = combo >> 1, q = combo & 1;
        const float inv = 1.0f / L;
        __half *dst = attn16 + static_cast<size_t>(it.t0 + it.qa + j) * QDIM + (2 * it.h + q) * HD + 4 * lane;
        *reinterpret_cast<__half2 *>(dst) = __floats2half2_rn(acc.x * inv, acc.y * inv);
        *reinterpret_cast<__half2 *>(dst + 2) = __floats2half2_rn(acc.z * inv, acc.w * inv);
    }
}

// ------------------------------------------------------------------ decode attention
//
// One new row per sequence (the decode steps of the talker and the
// predictor): split-K over the context.  One CTA per (sequence, kv head,
// split); the split's keys [ka, kb) (ka page-aligned) are visited in tiles of
// DSPLIT keys (4 pages): the K and V pages of a tile come in by bulk copies
// (16 positions x 128 of one head are contiguous in a page).  One buffer per
// CTA keeps shared memory at 33 KB (bf16), so that 6 CTAs share an SM and
// hide each other's copy latency.  Per tile, 128 threads score the 2 query
// heads x 64 keys, a shuffle softmax per head updates the running (m, l), and
// thread (head, dim pair) accumulates the output.  A single split writes the
// normalised row, several write (m, l, o) partials for attn_combine_kernel.
constexpr int DSPLIT = 64;
constexpr int DTHREADS = 128;
constexpr int DMAX_SPLITS = 16;  // fixed split count per sequence at most

template <class KVT>
struct DecodeSmem {
    KVT ks[DSPLIT][HD];
    KVT vs[DSPLIT][HD];
    float qs[2][HD];
    float p[2][DSPLIT];
    float red[4][2];
    uint64_t bar;
    int ok;
};

__device__ __forceinline__ float2 load2(const float *s) { return *reinterpret_cast<const float2 *>(s); }
__device__ __forceinline__ float2 load2(const __nv_bfloat16 *s) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(s));
}

template <class KVT>
__device__ __forceinline__ void decode_issue(DecodeSmem<KVT> *sm, const KVPool<KVT> &pool, int layer, int seq,
                                             int head, int k0, int nk) {
    constexpr uint32_t PAGE_BYTES = PAGE * HD * sizeof(KVT);
    const int npg = (nk + PAGE - 1) / PAGE;
    mbar_arrive_tx(&sm->bar, 2 * npg * PAGE_BYTES);
    for (int i = 0; i < npg; ++i) {
        const int pos = k0 + i * PAGE;
        bulk_g2s(&sm->ks[i * PAGE][0], kv_at(pool, layer, seq, pos, 0, head), PAGE_BYTES, &sm->bar);
        bulk_g2s(&sm->vs[i * PAGE][0], kv_at(pool, layer, seq, pos, 1, head), PAGE_BYTES, &sm->bar);
    }
}

template <class KVT>
__global__ void __launch_bounds__(DTHREADS) attn_decode_kernel(const AttnItem *items, const float *q32,
                                                              KVPool<KVT> pool, int layer, __half *attn16,
                                                              float *part, int *err) {
    extern __shared__ __align__(128) uint8_t dsm_raw[];
    DecodeSmem<KVT> *sm = reinterpret_cast<DecodeSmem<KVT> *>(dsm_raw);
    pdl_trigger();
    // the item (metadata copied before the call's first kernel) and, when
    // its first tile holds only cached positions (written by earlier calls,
    // which completed before this call's first copy), that tile's pages are
    // on their way before the previous kernel (the append of the new row)
    // has finished
    const AttnItem it = items[blockIdx.x];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q = tid >> 6, j = tid & 63;  // scores: (head, key); output: (head, dim pair j)
    const int nkeys = it.kb > it.ka ? it.kb - it.ka : 0;
    const int ntiles = (nkeys + DSPLIT - 1) / DSPLIT;
    const bool early = ntiles > 0 && it.ka + min(DSPLIT, nkeys) <= it.L0;
    if (tid == 0) {
        mbar_init(&sm->bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if (early) decode_issue(sm, pool, layer, it.seq, it.h, it.ka, min(DSPLIT, nkeys));
    }
    pdl_wait();
    if (tid == 0 && ntiles > 0 && !early) decode_issue(sm, pool, layer, it.seq, it.h, it.ka, min(DSPLIT, nkeys));
    for (int i = tid; i < 2 * HD / 4; i += DTHREADS) {
        const int hq = i / (HD / 4), d4 = i - hq * (HD / 4);
        store4(&sm->qs[hq][4 * d4], load4(q32 + static_cast<size_t>(it.t0) * QDIM + (2 * it.h + hq) * HD + 4 * d4));
    }
    __syncthreads();
    const float scale = 1.0f / sqrtf(static_cast<float>(HD));
    float m_run = -INFINITY, l_run = 0.f, ox = 0.f, oy = 0.f;
    int waited = 0;  // tiles whose copies are known to have landed (thread 0)
    for (int t = 0; t < ntiles; ++t) {
        const int k0 = it.ka + t * DSPLIT, nk = min(DSPLIT, it.kb - k0);
        if (tid == 0) {
            // tile t was issued before the loop (t = 0) or at the end of t-1
            const bool got = mbar_wait(&sm->bar, t & 1, nullptr);
            waited = got ? t + 1 : waited;
            sm->ok = got ? 1 : 0;
        }
        __syncthreads();  // (A) tile t landed (or not: uniform decision)
        if (!sm->ok) break;
        float sc = -INFINITY;
        if (j < nk) {
            // the dims from pair j on: the 32 keys of a warp hit 32 banks
            float a = 0.f;
#pragma unroll 8
            for (int e = 0; e < HD / 2; ++e) {
                const int pr = (e + j) & (HD / 2 - 1);
                const float2 kv2 = load2(&sm->ks[j][2 * pr]);
                const float2 qv2 = *reinterpret_cast<const float2 *>(&sm->qs[q][2 * pr]);
                a = fmaf(qv2.x, kv2.x, a);
                a = fmaf(qv2.y, kv2.y, a);
            }
            sc = a * scale;
        }
        float mt = sc;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
        if (lane == 0) sm->red[warp][0] = mt;
        __syncthreads();  // (B)
        const float m_new = fmaxf(m_run, fmaxf(sm->red[2 * q][0], sm->red[2 * q + 1][0]));
        const float e = j < nk ? expf(sc - m_new) : 0.f;
        float lt = e;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o);
        if (lane == 0) sm->red[warp][1] = lt;
        sm->p[q][j] = e;
        __syncthreads();  // (C)
        const float corr = expf(m_run - m_new);  // 0 on the first tile
        l_run = fmaf(l_run, corr, sm->red[2 * q][1] + sm->red[2 * q + 1][1]);
        ox *= corr;
        oy *= corr;
        for (int k = 0; k < nk; ++k) {
            const float pk = sm->p[q][k];
            const float2 v2 = load2(&sm->vs[k][2 * j]);
            ox = fmaf(pk, v2.x, ox);
            oy = fmaf(pk, v2.y, oy);
        }
        m_run = m_new;
        __syncthreads();  // (D) buffer, p and red free: the next tile comes in
        if (tid == 0 && t + 1 < ntiles) decode_issue(sm, pool, layer, it.seq, it.h, k0 + DSPLIT, min(DSPLIT, it.kb - k0 - DSPLIT));
    }
    if (tid == 0 && waited < ntiles) {
        // a wait gave up: report it, then wait (bounded) for the copy in
        // flight so that none lands after the CTA has exited
        atomicCAS(err, 0, ERR_TIMEOUT);
        mbar_wait(&sm->bar, waited & 1, nullptr);
    }
    if (it.part < 0) {
        const float inv = 1.0f / l_run;
        *reinterpret_cast<__half2 *>(attn16 + static_cast<size_t>(it.t0) * QDIM + (2 * it.h + q) * HD + 2 * j) =
            __floats2half2_rn(ox * inv, oy * inv);
    } else {
        float *pp = part + (static_cast<size_t>(it.part) * 2 + q) * PSTRIDE;
        *reinterpret_cast<float2 *>(pp + 2 * j) = make_float2(ox, oy);
        if (j == 0) {
            pp[HD] = m_run;
            pp[HD + 1] = l_run;
        }
    }
}

// The splits of one-row sequences: warp per (call, q head); items
// first[call*8 + h] .. +count of kv head h hold its partials.
__global__ void attn_combine_kernel(const int *first, const int *count, const int *tok, int ncalls, const float *part,
                                    __half *attn16) {
    pdl_trigger();
    pdl_wait();
    const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (w >= ncalls * HQ) return;
    const int call = w / HQ, qh = w - call * HQ, h = qh >> 1, q = qh & 1;
    const int f = first[call * HKV + h], n = count[call * HKV + h];
    if (n <= 0) return;
    float M = -INFINITY;
    for (int s = 0; s < n; ++s) M = fmaxf(M, part[(static_cast<size_t>(f + s) * 2 + q) * PSTRIDE + HD]);
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < n; ++s) {
        const float *pp = part + (static_cast<size_t>(f + s) * 2 + q) * PSTRIDE;
        const float e = pp[HD] == -INFINITY ? 0.f : expf(pp[HD] - M);
        L = fmaf(pp[HD + 1], e, L);
        const float4 v = load4(pp + 4 * lane);
        acc.x = fmaf(v.x, e, acc.x);
        acc.y = fmaf(v.y, e, acc.y);
        acc.z = fmaf(v.z, e, acc.z);
        acc.w = fmaf(v.w, e, acc.w);
    }
    const float inv = 1.0f / L;
    __half *dst = attn16 + static_cast<size_t>(tok[call]) * QDIM + qh * HD + 4 * lane;
    *reinterpret_cast<__half2 *>(dst) = __floats2half2_rn(acc.x * inv, acc.y * inv);
    *reinterpret_cast<__half2 *>(dst + 2) = __floats2half2_rn(acc.z * inv, acc.w * inv);
}

// ------------------------------------------------------------------ batched frames
//
// TQwenTalker.NextFrame (talker.pas:640-681) for many utterances: the
// per-utterance state lives on the device, the steps of a frame are batched
// forwards over all utterances (one predictor call per group, one talker
// call), and these kernels do the choices and the embedding sums between them.

// per-utterance frame state (TQwenTalker fields fHistory, fStep, ...)
struct SeqState {
    int next_code0;     // chosen at the end of the previous talker forward
    int done;           // next_code0 == eos
    int hist_len;       // frames returned (history length)
    int step;           // fStep
    int trailing_rows;  // rows of this utterance's trailing text
    int pad[3];
};

// Start: reset the state of seqs[i], clear its history marks.
__global__ void frames_start_kernel(const int *seqs, const int *trailing_rows, SeqState *ss, unsigned char *seen,
                                    int vocab) {
    pdl_trigger();
    pdl_wait();
    const int s = seqs[blockIdx.x];
    unsigned char *m = seen + static_cast<size_t>(s) * vocab;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) m[i] = 0;
    if (threadIdx.x == 0) {
        SeqState st = {};
        st.trailing_rows = trailing_rows[blockIdx.x];
        ss[s] = st;
    }
}

// Frame begin (talker.pas:656-667): code 0 joins the history; predictor
// input rows 2i, 2i+1 = [talker state, codec_emb[code 0]].
__global__ void frames_begin_kernel(const int *seqs, SeqState *ss, unsigned char *seen, int vocab,
                                    const float *hid, const float *codec_emb, float *px, int *codes, int groups) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x, s = seqs[i];
    const int c0 = ss[s].next_code0;
    const float *h = hid + static_cast<size_t>(s) * H;
    const float *e = codec_emb + static_cast<size_t>(c0) * H;
    float *x0 = px + static_cast<size_t>(2 * i) * H;
    for (int c = threadIdx.x; c < H / 4; c += blockDim.x) {
        store4(x0 + 4 * c, load4(h + 4 * c));
        store4(x0 + H + 4 * c, load4(e + 4 * c));
    }
    if (threadIdx.x == 0) {
        seen[static_cast<size_t>(s) * vocab + c0] = 1;
        ss[s].hist_len += 1;
        codes[i * groups] = c0;
    }
}

// block-wide argmax key of n values
__device__ __forceinline__ unsigned long long block_argmax(unsigned long long b, unsigned long long *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
        b = t > b ? t : b;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = b;
    __syncthreads();
    if (threadIdx.x < 32) {
        b = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
            b = t > b ? t : b;
        }
        if (threadIdx.x == 0) red[0] = b;
    }
    __syncthreads();
    return red[0];
}

// ChooseCode (talker.pas:632-638), greedy, after predictor step g: code g+1
// of row i = the first maximum of its logits; the next predictor input row
// is pred_emb[g][code] (talker.pas:670-675).
//  samp.on: the code is drawn (draw (frame, g + 1) of the utterance's
//  stream seed + s), else the first maximum; 256 threads.
__global__ void __launch_bounds__(256) frames_pred_argmax_kernel(const float *logits, int vocab, int g, int groups,
                                                                 const float *pred_emb, float *px, int *codes,
                                                                 const int *seqs, const SeqState *ss,
                                                                 SampleParams samp, unsigned long long seed) {
    pdl_trigger();
    pdl_wait();
    __shared__ unsigned long long red[32];
    __shared__ SampleScratch scr;
    const int i = blockIdx.x;
    const float *lg = logits + static_cast<size_t>(i) * vocab;
    int code;
    if (samp.on) {
        const int s = seqs[i];
        code = sample_draw<256>([&](int j) { return lg[j]; }, vocab, samp,
                                sample_uniform(seed + static_cast<unsigned long long>(s), ss[s].step, g + 1), &scr,
                                static_cast<int>(threadIdx.x));
    } else {
        unsigned long long b = 0ull;
        for (int j = threadIdx.x; j < vocab; j += blockDim.x) {
            const unsigned long long k = argkey(lg[j], j);
            b = k > b ? k : b;
        }
        code = key_index(block_argmax(b, red));
    }
    if (threadIdx.x == 0) codes[i * groups + g + 1] = code;
    if (g + 1 < groups - 1) {
        const float *e = pred_emb + (static_cast<size_t>(g) * vocab + code) * H;
        float *x = px + static_cast<size_t>(i) * H;
        for (int c = threadIdx.x; c < H / 4; c += blockDim.x) store4(x + 4 * c, load4(e + 4 * c));
    }
}

// The next talker input (talker.pas:669-677): codec_emb[code 0] + the 15
// predictor embeddings in group order + trailing[step] (tts_pad after the
// trailing rows), summed left to right in float32.
__global__ void frames_talker_in_kernel(const int *seqs, const SeqState *ss, const int *codes, int groups,
                                        const float *codec_emb, const float *pred_emb, int pvocab,
                                        const float *const *trailing, const float *tts_pad, float *xt) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x, s = seqs[i];
    const int *cd = codes + i * groups;
    const int step = ss[s].step;
    const float *tr = step < ss[s].trailing_rows ? trailing[s] + static_cast<size_t>(step) * H
                                                 : tts_pad + static_cast<size_t>(s) * H;
    for (int c = threadIdx.x; c < H / 4; c += blockDim.x) {
        float4 a = load4(codec_emb + static_cast<size_t>(cd[0]) * H + 4 * c);
        for (int g = 1; g < groups; ++g) {
            const float4 e = load4(pred_emb + (static_cast<size_t>(g - 1) * pvocab + cd[g]) * H + 4 * c);
            a = make_float4(a.x + e.x, a.y + e.y, a.z + e.z, a.w + e.w);
        }
        const float4 e = load4(tr + 4 * c);
        store4(xt + static_cast<size_t>(i) * H + 4 * c, make_float4(a.x + e.x, a.y + e.y, a.z + e.z, a.w + e.w));
    }
}

// ChooseCode0 (talker.pas:595-630), greedy, after a talker forward: the
// last 1024 ids forbidden but eos, eos forbidden before 2 frames, the
// repetition penalty once per distinct code of the history; the normed
// state of the row becomes the utterance's talker state.  done[i] = eos
// chosen (read by the host).  start != 0: after the prefill (empty history).
//  samp0.on: code 0 is drawn (draw (frame, 0) of the utterance's stream
//  seed + s; frame = the index of the frame the code belongs to), else the
//  first maximum; 256 threads.
__global__ void __launch_bounds__(256) frames_choose0_kernel(const int *seqs, const float *logits, const float *hidden,
                                                             int vocab, int eos, float penalty,
                                                             const unsigned char *seen, SeqState *ss, float *hid,
                                                             int *done, int start, SampleParams samp0,
                                                             unsigned long long seed) {
    pdl_trigger();
    pdl_wait();
    __shared__ unsigned long long red[32];
    __shared__ SampleScratch scr;
    const int i = blockIdx.x, s = seqs[i];
    const float *lg = logits + static_cast<size_t>(i) * vocab;
    const unsigned char *m = seen + static_cast<size_t>(s) * vocab;
    const int hist = ss[s].hist_len;
    // ChooseCode0's processors (talker.pas:595-625)
    auto value = [&](int j) {
        float w = lg[j];
        if (j >= vocab - 1024 && j != eos) w = -INFINITY;
        else if (j == eos && hist < 2) w = -INFINITY;
        else if (penalty != 1.0f && m[j]) w = w > 0.f ? __fdiv_rn(w, penalty) : w * penalty;
        return w;
    };
    int code;
    if (samp0.on) {
        const int frame = start ? 0 : ss[s].step + 1;
        code = sample_draw<256>(value, vocab, samp0, sample_uniform(seed + static_cast<unsigned long long>(s), frame, 0),
                                &scr, static_cast<int>(threadIdx.x));
    } else {
        unsigned long long b = 0ull;
        for (int j = threadIdx.x; j < vocab; j += blockDim.x) {
            const unsigned long long k = argkey(value(j), j);
            b = k > b ? k : b;
        }
        code = key_index(block_argmax(b, red));
    }
    for (int c = threadIdx.x; c < H / 4; c += blockDim.x)
        store4(hid + static_cast<size_t>(s) * H + 4 * c, load4(hidden + static_cast<size_t>(i) * H + 4 * c));
    if (threadIdx.x == 0) {
        ss[s].next_code0 = code;
        ss[s].done = code == eos ? 1 : 0;
        if (!start) ss[s].step += 1;
        done[i] = code == eos ? 1 : 0;
    }
}

// ------------------------------------------------------------------ prefill attention (tensor cores)
//
// Causal attention of long runs of new rows (prefill) on the 5th-generation
// tensor cores, flash-attention style.  One CTA per (sequence, kv head,
// block of up to 128 new rows) takes both query heads of the kv head, so
// each K/V tile is read once for the two.
//  - K and V come from the fp16 mirror of the pages (written by the QKV
//    epilogue beside the cache, each page already in the tensor cores'
//    layout): warp 8 brings the 8 pages of a 128-key tile into one of two
//    buffers with one bulk copy per page and K/V (tile t + 1 lands while
//    tile t is in the products and the softmax), and clears the V rows of
//    the pages past the causal end.  A tile is [8-key group][64-dim
//    atom][8 rows x 128 bytes]: K is a K-major operand with 8-row groups
//    2048 bytes apart and the second dim atom 1024 bytes on; V is the
//    MN-major B operand of P V (dim atoms 1024 bytes apart, key groups 2048),
//    so nothing is transposed or converted.
//  - Q of both heads is converted to fp16 by warps 0-7 into the A-operand
//    layout (rows of 128 bytes, the two 64-dim atoms 16 KB apart).
//  - warps 0-7: thread 128 g + r owns query row r of head 2h + g.  S_g =
//    Q_g K^T (8 x tcgen05.mma, M 128, N 128, K 16) lands in TMEM columns
//    [128 g, +128); row r is read back by its thread (warps 4g..4g+3 reach
//    TMEM lanes 0-127), masked causally on the diagonal tile, its running
//    (max, sum) updated in f32, its row of O_g rescaled in TMEM when the
//    maximum moved, and P_g = exp(S - max) written as fp16 in the A-operand
//    layout (P_0 over the consumed K tile, P_1 in its own tile); then O_g +=
//    P_g V into columns [256 + 128 g, +128).  After the last tile, O_g / sum
//    goes to attn16 as fp16.
//  - 512 TMEM columns and 225 KB of shared memory: one CTA per SM.
//  - every mbarrier wait is bounded; a timeout sets the error word, and the
//    MMA thread waits (bounded) for its own products before TMEM is freed.
constexpr int TA_ROWS = 128;   // query rows per CTA and head (MMA M)
constexpr int TA_KEYS = 128;   // keys per tile (MMA N of S, K of P V)
constexpr int TA_CONSUMERS = 256;  // warps 0-7
constexpr int TA_THREADS = TA_CONSUMERS + 32;  // + warp 8: the copies
constexpr int TC_MIN_ROWS = 32;  // sequences with more new rows than this use this kernel
constexpr int TA_TILE = TA_ROWS * HD * 2;  // 32 KB: one fp16 operand tile

struct __align__(1024) TaSmem {
    uint8_t q[2][TA_TILE];
    uint8_t kp[2][TA_TILE];  // buffer b: the K tile (8 mirror pages), then (once both S are computed) P of head 0
    uint8_t v[2][TA_TILE];   // buffer b: the V tile (8 mirror pages)
    uint8_t p1[TA_TILE];     // P of head 1
    uint64_t kv_full[2];     // the copies' bytes (one arrival: warp 8)
    uint64_t kv_free[2];     // tcgen05.commit after the P V products that read buffer b
    uint64_t s_done, o_done, fin;
    uint32_t tmem_base;
};
static_assert(sizeof(TaSmem) + 1024 <= 232448, "prefill attention: shared memory above 227 KB");

// byte offset of element (row, kk) of a 128 x 128 fp16 operand tile in the
// K-major 128B-swizzle layout (atoms of 64 K elements, 16 KB each)
__device__ __forceinline__ uint32_t ta_off(int row, int kk) {
    const int a = kk >> 6, c = kk & 63, j = c >> 3;
    return a * (TA_ROWS * 128) + (row >> 3) * 1024 + (row & 7) * 128 + ((j ^ (row & 7)) << 4) + (c & 7) * 2;
}
// store 8 consecutive K elements (one 16-byte chunk) of row `row` from kk
__device__ __forceinline__ void ta_store8(uint8_t *tile, int row, int kk, const float *v) {
    __half2 h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4 *>(tile + ta_off(row, kk)) = *reinterpret_cast<uint4 *>(h);
}

// store 4 consecutive elements (half a 16-byte chunk) of row `row` from kk (kk % 4 == 0)
__device__ __forceinline__ void ta_store4(uint8_t *tile, int row, int kk, float4 v) {
    const __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t *>(&a);
    u.y = *reinterpret_cast<const uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(tile + ta_off(row, kk)) = u;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float *v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
        "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
        "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
        "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
        : "memory");
}

// a 128B-swizzle shared-memory descriptor with explicit leading and stride
// byte offsets
__device__ __forceinline__ uint64_t umma_desc_sw128_at(const void *smem, uint32_t lbo, uint32_t sbo) {
    return ((smem_u32(smem) >> 4) & 0x3FFFull) | (static_cast<uint64_t>(lbo >> 4) << 16) |
           (static_cast<uint64_t>(sbo >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// thread 0: S = Q K^T for one 128-key tile (8 MMAs, K = 16 each).  Q (128
// rows x 128 dims) is the K-major A operand, its two 64-dim atoms 16 KB
// apart; K (8 mirror pages) is the K-major B operand, 8-key groups 2048
// bytes apart and the second dim atom 1024 bytes on; a K = 16 step moves 32
// bytes inside an atom.
__device__ __forceinline__ void ta_mma_s(uint32_t tmem_d, const uint8_t *q, const uint8_t *k) {
    const uint32_t idesc = umma_idesc_f16(TA_ROWS, TA_KEYS);
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
        const uint64_t da = umma_desc_sw128(q + (kk >> 2) * (TA_ROWS * 128)) + 2 * (kk & 3);
        const uint64_t db = umma_desc_sw128_at(k + (kk >> 2) * 1024, 16, 2048) + 2 * (kk & 3);
        umma_f16(tmem_d, da, db, idesc, kk > 0 ? 1u : 0u);
    }
}

// thread 0: O += P V for one 128-key tile.  P (128 rows x 128 keys) is the
// K-major A operand (atoms 16 KB apart); V (8 mirror pages: 128 keys x 128
// dims) is the MN-major B operand, its dim atoms 1024 bytes apart (leading
// byte offset) and 8-key groups 2048 apart (stride byte offset); a K = 16
// step moves two key groups, 4096 bytes.
__device__ __forceinline__ void ta_mma_pv(uint32_t tmem_d, const uint8_t *p, const uint8_t *v, bool accumulate) {
    const uint32_t idesc = umma_idesc_f16(TA_ROWS, HD) | (1u << 16);  // B MN-major
#pragma unroll
    for (int kk = 0; kk < TA_KEYS / 16; ++kk) {
        const uint64_t da = umma_desc_sw128(p + (kk >> 2) * (TA_ROWS * 128)) + 2 * (kk & 3);
        const uint64_t db = umma_desc_sw128_at(v + 4096 * kk, 1024, 2048);
        umma_f16(tmem_d, da, db, idesc, (accumulate || kk > 0) ? 1u : 0u);
    }
}
static_assert(PAGE == 16 && TA_KEYS == 8 * PAGE && TA_TILE == 8 * KV16_PAGE,
              "a key tile is 8 mirror pages of K (and 8 of V)");

// consumer warps only: bar.sync on barrier 1 that also ORs a flag over them
__device__ __forceinline__ bool ta_consumers_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v)), "n"(TA_CONSUMERS)
        : "memory");
    return r != 0;
}

template <class KVT>
__global__ void __launch_bounds__(TA_THREADS, 1) attn_prefill_tc_kernel(const AttnItem *items, const float *q32,
                                                                       KVPool<KVT> pool, const __half *kv16, int layer,
                                                                       __half *attn16, int *err) {
    extern __shared__ __align__(1024) uint8_t ta_raw[];
    TaSmem *sm = reinterpret_cast<TaSmem *>((reinterpret_cast<uintptr_t>(ta_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sm->kv_full[b], 1);
            mbar_init(&sm->kv_free[b], 1);
        }
        mbar_init(&sm->s_done, 1);
        mbar_init(&sm->o_done, 1);
        mbar_init(&sm->fin, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {  // S_g: columns [128 g, 128 g + 128), O_g: [256 + 128 g, ...)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&sm->tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pdl_trigger();
    pdl_wait();
    const AttnItem it = items[blockIdx.x];
    const int h = it.h;                  // kv head
    const int nq = it.qb - it.qa;        // 1..128 rows
    const int kend = it.L0 + it.qb;      // keys [0, kend) (causal)
    const int ntiles = (kend + TA_KEYS - 1) / TA_KEYS;
    if (warp < 8) {
        // Q: warp w takes rows [32 (w % 4), +32) of head 2h + w / 4, one row
        // per load (lane l: dims 4l..4l+3), 16 loads in flight
        const int wg = warp >> 2, wr = 32 * (warp & 3);
        const float *src = q32 + static_cast<size_t>(it.t0 + it.qa) * QDIM + (2 * h + wg) * HD + 4 * lane;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            float4 qb[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int row = wr + 16 * half + i;
                qb[i] = row < nq ? load4(src + static_cast<size_t>(row) * QDIM) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) ta_store4(sm->q[wg], wr + 16 * half + i, 4 * lane, qb[i]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tm = sm->tmem_base;
    if (warp == 8) {
        // ---- copies: tile t into buffer t % 2 once the P V products of
        // tile t - 2 (the last to read it) are complete: one bulk copy of 4 KB
        // per mirror page and K/V; the V rows of pages past the causal end
        // are cleared (P is 0 there, and 0 times a stale NaN is NaN)
        int issued = 0;
        for (int t = 0; t < ntiles; ++t) {
            const int b = t & 1, kt = t * TA_KEYS;
            if (t >= 2 && !mbar_wait(&sm->kv_free[b], ((t >> 1) - 1) & 1, nullptr)) {
                if (lane == 0) atomicCAS(err, 0, ERR_TIMEOUT);
                break;
            }
            issued = t + 1;
            const int npg = min(TA_KEYS / PAGE, (kend - kt + PAGE - 1) / PAGE);  // pages holding keys < kend
            for (int i = npg * KV16_PAGE / 16 + lane; i < TA_TILE / 16; i += 32)
                reinterpret_cast<uint4 *>(sm->v[b])[i] = make_uint4(0u, 0u, 0u, 0u);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_tx(&sm->kv_full[b], static_cast<uint32_t>(npg * 2 * KV16_PAGE));
                for (int pg = 0; pg < npg; ++pg) {
                    const int page = pool.pages[it.seq * pool.mpps + (kt >> 4) + pg];
                    const uint8_t *k = reinterpret_cast<const uint8_t *>(kv16) +
                                       kv16_page_index(page, pool.layers, layer, 0, h) * KV16_PAGE;
                    const uint8_t *v = reinterpret_cast<const uint8_t *>(kv16) +
                                       kv16_page_index(page, pool.layers, layer, 1, h) * KV16_PAGE;
                    bulk_g2s(sm->kp[b] + pg * KV16_PAGE, k, KV16_PAGE, &sm->kv_full[b]);
                    bulk_g2s(sm->v[b] + pg * KV16_PAGE, v, KV16_PAGE, &sm->kv_full[b]);
                }
            }
        }
        // no copy may land after the CTA is gone (the consumers may have
        // stopped early): wait (bounded) for the last one issued into each
        // buffer; the earlier ones were consumed before their buffer refilled
        if (lane == 0)
            for (int t = issued > 2 ? issued - 2 : 0; t < issued; ++t)
                mbar_wait(&sm->kv_full[t & 1], (t >> 1) & 1, nullptr);
    } else {
        // ---- consumers
        const int g = tid >> 7, r = tid & (TA_ROWS - 1);  // query head 2h + g, row r
        const int qh = 2 * h + g;
        const int qpos = it.L0 + it.qa + r;
        const uint32_t tm_s = tm + TA_KEYS * g, tm_o = tm + 2 * TA_KEYS + HD * g;
        const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
        const float sl2 = (1.0f / sqrtf(static_cast<float>(HD))) * 1.44269504088896341f;  // scale log2(e)
        float m_run = -INFINITY, l_run = 0.f;  // running maximum of the raw scores, sum of exponentials
        bool failed = false;
        for (int t = 0; t < ntiles; ++t) {
            const int b = t & 1, kt = t * TA_KEYS;
            bool good = true;
            if (tid == 0) {
                // S_0, S_1 of tile t once it has landed (S's TMEM columns were
                // read by every consumer before the last consumer barrier)
                good = mbar_wait(&sm->kv_full[b], (t >> 1) & 1, nullptr);
                if (good) {
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    ta_mma_s(tm, sm->q[0], sm->kp[b]);
                    ta_mma_s(tm + TA_KEYS, sm->q[1], sm->kp[b]);
                    umma_commit(&sm->s_done);
                }
            }
            good = mbar_wait(&sm->s_done, t & 1, nullptr) && good;
            __syncwarp();
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            // row maximum of the raw scores (first pass over TMEM; scale > 0,
            // so it gives the maximum of the scaled ones).  Only a tile with a
            // key past the block's first row is masked; four partial maxima
            // (and sums below) keep the dependency chains short
            const bool diag = kt + TA_KEYS - 1 > it.L0 + it.qa;
            float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            for (int c = 0; c < TA_KEYS; c += 32) {
                float sv[32];
                tmem_ld32(tm_s + lane_base + c, sv);
                if (diag) {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (kt + c + j <= qpos) mx[j & 3] = fmaxf(mx[j & 3], sv[j]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) mx[j & 3] = fmaxf(mx[j & 3], sv[j]);
                }
            }
            const float m_new = fmaxf(m_run, fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])));
            // exp(scale (s - m)) = exp2(s sl2 - m sl2), sl2 = scale log2(e)
            const float ms = m_new * sl2;
            const float corr = exp2f(fmaf(m_run, sl2, -ms));  // 0 on the first tile (m_run = -inf)
            // P_1's tile and the O accumulator: tile t - 1's P V products are
            // complete (P_0 goes over this tile's K: both S products are done)
            if (t > 0) good = mbar_wait(&sm->o_done, (t - 1) & 1, nullptr) && good;
            __syncwarp();
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            uint8_t *ptile = g == 0 ? sm->kp[b] : sm->p1;
            // P = exp(S - m), second pass over TMEM; row sum
            float ls[4] = {0.f, 0.f, 0.f, 0.f};
            for (int c = 0; c < TA_KEYS; c += 32) {
                float sv[32];
                tmem_ld32(tm_s + lane_base + c, sv);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    float e = exp2f(fmaf(sv[j], sl2, -ms));
                    if (diag && kt + c + j > qpos) e = 0.f;
                    sv[j] = e;
                    ls[j & 3] += e;
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) ta_store8(ptile, r, c + 8 * q, sv + 8 * q);
            }
            l_run = fmaf(l_run, corr, (ls[0] + ls[1]) + (ls[2] + ls[3]));
            m_run = m_new;
            // rescale this row of the O accumulator, unless no row of the
            // warp has a new maximum (TMEM loads and stores are warp-wide)
            if (t > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
                for (int c = 0; c < HD; c += 32) {
                    float ov[32];
                    tmem_ld32(tm_o + lane_base + c, ov);
#pragma unroll
                    for (int j = 0; j < 32; ++j) ov[j] *= corr;
                    tmem_st32(tm_o + lane_base + c, ov);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            if (ta_consumers_or(!good)) {
                failed = true;
                break;
            }
            if (tid == 0) {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                ta_mma_pv(tm + 2 * TA_KEYS, sm->kp[b], sm->v[b], t > 0);
                ta_mma_pv(tm + 2 * TA_KEYS + HD, sm->p1, sm->v[b], t > 0);
                umma_commit(&sm->o_done);
                umma_commit(&sm->kv_free[b]);  // the loaders may refill buffer b
            }
        }
        if (!failed && !mbar_wait(&sm->o_done, (ntiles - 1) & 1, nullptr)) failed = true;
        __syncwarp();
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // O / sum of row r to attn16 (the TMEM loads are warp-wide: every lane
        // takes part, the rows beyond the block only skip the store)
        const float inv = 1.0f / l_run;
        __half *dst = attn16 + static_cast<size_t>(it.t0 + it.qa + (r < nq ? r : 0)) * QDIM + qh * HD;
        for (int c = 0; c < HD; c += 32) {
            float ov[32];
            tmem_ld32(tm_o + lane_base + c, ov);
            if (!failed && r < nq) {
#pragma unroll
                for (int j = 0; j < 32; j += 2)
                    *reinterpret_cast<__half2 *>(dst + c + j) = __floats2half2_rn(ov[j] * inv, ov[j + 1] * inv);
            }
        }
        if (failed) atomicCAS(err, 0, ERR_TIMEOUT);
    }
    // the MMA thread waits (bounded) for every product it issued, then TMEM
    // is freed
    if (tid == 0) {
        umma_commit(&sm->fin);
        if (!mbar_wait(&sm->fin, 0, nullptr)) atomicCAS(err, 0, ERR_TIMEOUT);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tm) : "memory");
    }
}

}  // namespace qtts
