// qtts_decode.cuh -- the persistent decode kernel of libqtts (sm_100a).
//
// One cooperative launch runs either one TQwenLm.Forward of <= RMAX rows
// (mormot.ai.tts.qwen.lm.pas:391-408) or one whole TQwenTalker.NextFrame
// (mormot.ai.tts.qwen.talker.pas:640-681): 15 code-predictor steps with their
// heads and greedy argmax, the sum of the 16 code embeddings, the talker step,
// its head and ChooseCode0 for the next frame.
//
// Shape of the kernel
//  - one CTA per SM (grid = SM count, ~206 KB shared memory each), 16 warps:
//    warps 0..14 compute, warp 15 is the weight producer.
//  - the producer walks the same program as the compute warps and streams
//    this CTA's slice of every weight matrix, in program order, through a
//    ring of NSTAGES shared-memory stages with cp.async.bulk (global ->
//    shared, mbarrier complete_tx).  Weights never depend on activations, so
//    the stream runs ahead across grid barriers: the next matrix is already
//    in shared memory when its activations become ready.
//  - the compute warps run the phases of each layer, separated by grid
//    barriers (monotonic counter, red.release / ld.acquire, bounded spin):
//      P1 rmsnorm + QKV GEMV -> qkv; then this CTA's cached K/V tile for P2
//         is prefetched into shared memory (cp.async.bulk) before the barrier
//      P2 q/k-norm + RoPE + KV append, attention over one split of the
//         context (positions spread over the warps) -> partials (o, max, sum)
//      P3 combine the partials of all heads + O GEMV + residual
//      P4 rmsnorm + gate/up GEMV + SiLU*up -> act
//      P5 down GEMV + residual
//    then the final rmsnorm + head GEMV + argmax.  Each CTA keeps its slice
//    of the residual stream in shared memory (its O/down rows).
//  - every wait is bounded (%globaltimer); on timeout the kernel records
//    QTTS_E_TIMEOUT in the error word, waits (bounded) for its own bulk copies
//    in flight and returns.
//
// Weight layout on the device (bytes per row are multiples of 16):
//  - F32: [rows][K] float32.
//  - Q8_0 (row-packed): [K int8 quants][K/32 fp16 scales] per row: the same
//    34 bytes per 32 weights as ggml's block_q8_0, planar within the row so
//    that 128-bit loads and bulk copies stay aligned.
//  - QKV rows: q (2048), k (1024), v (1024); gate/up rows interleaved
//    (gate j at 2j, up j at 2j+1) so a CTA owns whole SwiGLU pairs.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "qtts_sample.cuh"

namespace qtts {

constexpr int H = 1024;                     // hidden
constexpr int HQ = 16;                      // query heads
constexpr int HKV = 8;                      // KV heads
constexpr int HD = 128;                     // head dim
constexpr int INTER = 3072;                 // SwiGLU intermediate
constexpr int QDIM = HQ * HD;               // 2048
constexpr int KVDIM = HKV * HD;             // 1024
constexpr int QKV_ROWS = QDIM + 2 * KVDIM;  // 4096
constexpr int GU_ROWS = 2 * INTER;          // 6144
constexpr int RMAX = 4;                     // rows per launch
constexpr int MAX_GROUPS = 16;              // codes per frame

constexpr int NWARPS = 16;
constexpr int NTHREADS = NWARPS * 32;
constexpr int NCW = NWARPS - 1;  // compute warps
constexpr int NCT = NCW * 32;    // compute threads
constexpr int PRODUCER_WARP = NWARPS - 1;

constexpr int STAGE_BYTES = 24576;
constexpr int NSTAGES = 5;
constexpr int ACT_FLOATS = RMAX * INTER;  // staged activations [R][K]
constexpr int MAX_PARTS = 64;             // (row, K segment) partial sums of a CTA slice (grid >= 128)
constexpr int KO = 2 * HD;                // O-projection columns of one kv head (its 2 query heads)
constexpr int QKV_HEAD = 4 * HD;          // QKV rows of one kv head: q(2h), q(2h+1), k(h), v(h)
constexpr int BAR_WORDS = 16;             // barrier counters: [0] grid, [1] exit (the rest reserved)
constexpr int PSTRIDE = 132;              // attention partial: o[128], m, l
constexpr int ATT_TILE = 32;              // context positions per attention tile
constexpr int XS_MAX = 16;                // residual rows owned by a CTA (grid >= 64)

constexpr int WDT_F32 = 0;
constexpr int WDT_Q8 = 1;

constexpr int ERR_TIMEOUT = 5;
constexpr int ERR_CAPACITY = 4;

// every wait gives up after this many SM cycles (about 2 s at B200 clocks);
// clock64() is local to the SM and cheap, unlike %globaltimer
constexpr long long WAIT_CYCLES = 4000000000ll;

__host__ __device__ constexpr int row_bytes(int wdt, int k) { return wdt == WDT_F32 ? k * 4 : k + k / 16; }

// the CTAs of a grid of g are split into HKV contiguous groups, one per kv
// head: CTA b belongs to head (b * HKV) / g, index j of nj in its group
__host__ __device__ inline void head_group(int b, int g, int &h, int &j, int &nj) {
    h = (b * HKV) / g;
    const int g0 = (h * g + HKV - 1) / HKV, g1 = ((h + 1) * g + HKV - 1) / HKV;
    j = b - g0;
    nj = g1 - g0;
}

// contexts of at most one attention tile take the per-head path (attention
// of a kv head in every CTA of its group, fused with the O projection)
__host__ __device__ inline bool per_head_path(int T) { return T <= ATT_TILE; }

// attention splits of a context of T positions over a grid of g CTAs
__host__ __device__ inline int att_splits(int T, int g) {
    int s = (T + ATT_TILE - 1) / ATT_TILE;
    int cap = g / HKV;
    s = s < cap ? s : cap;
    return s < 1 ? 1 : s;
}

// ------------------------------------------------------------------ descriptors

struct DLayer {
    const uint8_t *wqkv, *wo, *wgu, *wd;
    // batch-1 kernel layouts: QKV rows by kv head [HKV][q(2h) q(2h+1) k(h) v(h)][H],
    // the O projection by kv head [HKV][H rows][KO columns]
    const uint8_t *wqkvh, *woh;
    const float *in_norm, *post_norm, *q_norm, *k_norm;
};

struct DStack {
    const DLayer *layer;  // device array
    int layers;
    float eps;
    const float *final_norm;
    int keep_l2;  // stream with L2 evict_last (weights that fit in L2)
};

struct DCtx {      // KV cache [layers][HKV][max_pos][HD], float32 or (kv16) fp16
    void *k, *v;
    int max_pos;
    int kv16;      // the cache holds half floats (TQwenLm's aKvF16)
};
// bytes of one cached K or V element
__host__ __device__ inline int kv_bytes(const DCtx &c) { return c.kv16 ? 2 : 4; }

// scratch of one runner (one lm or one talker), all in global memory
struct Scratch {
    float *x;       // [RMAX][H] residual stream
    // tagged handoffs: 64-bit words (tag << 32 | float bits), read by
    // polling until the word carries the tag of the handoff (no barrier)
    unsigned long long *x8;   // [RMAX][H] residual stream after the down projection
    unsigned long long *qkv;  // [RMAX][QKV_ROWS] QKV rows
    float *act;     // [RMAX][INTER]
    float *part;    // [HKV*maxS][RMAX][2][PSTRIDE] attention partials, or (per-head path)
                    // [RMAX][HKV * H] O-projection partials, one H-vector per kv head
    unsigned long long *arg;  // [grid] argmax keys
    unsigned *bar;  // [BAR_WORDS]: [0] grid barrier, [1] exit
    int *err;       // [0] error code, [1] where
    float *logits;  // [max head rows]
    float *hidden;  // [H] normed state of the last row
    float *xt;      // [H] talker input being summed (frame mode)
};

// device state of the frame loop (TQwenTalker fields fHistory, fStep, ...)
struct FrameState {
    int next_code0;  // chosen at the end of the previous talker forward
    int done;        // next_code0 == eos
    int hist_len;    // frames returned
    int step;        // fStep
    int tlen;        // talker cache length
    int codes[MAX_GROUPS];
    int pad[3];
};

struct Job {
    int mode;  // 0 = forward, 1 = frame
    // forward
    DStack st;
    DCtx ctx;
    const float *xin;  // [rows][H] device
    int rows, L0;
    const uint8_t *head_w;  // NULL: no head
    int head_rows;
    // frame
    DStack tst, pst;
    DCtx tctx, pctx;
    const uint8_t *theads;
    int tvocab;
    const uint8_t *const *pheads;  // device array [groups-1]
    int pvocab, groups;
    const float *codec_emb;  // [tvocab][H]
    const float *pred_emb;   // [groups-1][pvocab][H]
    const float *trailing;   // [trailing_rows][H]
    int trailing_rows;
    const float *tts_pad;    // [H]
    int eos;
    float penalty;
    unsigned char *seen;     // [tvocab] codes already returned
    // TQwenSampling (talker.pas:59-73): code 0 and the predictor's codes;
    // draw (frame, group) of the stream `seed`
    SampleParams samp0, samp;
    unsigned long long seed;
    FrameState *fs;
    int *codes_hist;         // [cap][groups] codes by frame index (may be NULL)
    int codes_cap;
    // phase timestamps of CTA 0 (profiling; NULL = off): (tag << 48) | ns
    unsigned long long *trace;
    int trace_cap;
    int *trace_n;
    // both
    Scratch s;
    const float *rope_cos, *rope_sin;  // [rope_pos][HD/2]
    int rope_pos;
    // the bound of the grid barrier and tagged-word spins (cycles;
    // WAIT_CYCLES unless a failure-path test shortens it), and arrivals the
    // grid barrier expects beyond the grid (0; a test sets 1: an arrival
    // that never comes)
    long long wait_cycles;
    int bar_extra;
    // launch epoch (1 .. 2^22 - 1): the high bits of every handoff tag, so
    // that no word left by an earlier launch carries a tag this one expects
    unsigned epoch;
};
constexpr unsigned EPOCH_LIMIT = 1u << 22;  // the host clears the tagged words before reusing epoch 1
constexpr int TAG_SEQ_BITS = 10;            // handoffs per launch < 1024 (a frame of 28 + 15 x 5 layers: 206)

// ------------------------------------------------------------------ PTX helpers

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// non-blocking test of an mbarrier phase (no suspension)
__device__ __forceinline__ bool mbar_test_now(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait on an mbarrier phase; false on timeout
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, const volatile int *abort_flag) {
    if (mbar_test(b, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_test(b, parity)) {
        if (abort_flag && *abort_flag) return false;
        if (clock64() - t0 > WAIT_CYCLES) return false;
    }
    return true;
}
__device__ __forceinline__ uint64_t l2_policy(bool keep) {
    uint64_t p;
    if (keep)
        asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    else
        asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// global -> shared bulk copy (no multicast); 16-byte aligned, size % 16 == 0
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// sums of a and b over the warp with 5 shuffles: lane 0 gets sum(a), lane 16 sum(b)
__device__ __forceinline__ float warp_sum2(float a, float b, int lane) {
    const bool hi = lane & 16;
    float keep = hi ? b : a, send = hi ? a : b;
    keep += __shfl_xor_sync(0xffffffffu, send, 16);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
    return keep;
}

// int8 x4 (one 32-bit word) -> 4 exact floats: byte b^0x80 placed in the
// mantissa of 2^23, minus 2^23+128
__device__ __forceinline__ float4 dq4(uint32_t w) {
    const uint32_t u = w ^ 0x80808080u;
    return make_float4(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f,
                       __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f,
                       __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f,
                       __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f);
}

// orderable key: larger value first, then smaller index (first maximum)
__device__ __forceinline__ unsigned long long argkey(float v, int idx) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(idx));
}
__device__ __forceinline__ int key_index(unsigned long long k) {
    return static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull));
}

// loads through L2 (data written by other CTAs in this launch: this SM's L1
// may hold an older copy)
__device__ __forceinline__ float4 ldcg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }

// tagged words of a handoff: one 8-byte access carries the value and its tag
__device__ __forceinline__ void st_tagged(unsigned long long *p, float v, unsigned tag) {
    const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void ld_tagged2(const unsigned long long *p, unsigned long long &a, unsigned long long &b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ bool tag_is(unsigned long long w, unsigned tag) {
    return static_cast<unsigned>(w >> 32) == tag;
}
// 4 halves (8-byte aligned, shared memory) -> float4
__device__ __forceinline__ float4 h4_to_f4(const __half *p) {
    const uint2 u = *reinterpret_cast<const uint2 *>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

// programmatic dependent launch: a kernel launched with programmatic stream
// serialisation may start while its predecessor runs; pdl_wait() returns
// once the predecessor grid has completed and its writes are visible (at
// once without such a launch), pdl_trigger() lets the successor launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------ shared memory

// Matrix phases in program order.  The producer and the compute warps walk
// the same order; it must not depend on data.  The matrices before M_HEAD
// have a fixed shape (their slices are computed once per launch).
enum Mat { M_QKV, M_O, M_OH, M_GU, M_D, M_HEAD };
constexpr int M_FIXED = M_HEAD;

struct __align__(128) Smem {
    uint8_t ring[NSTAGES][STAGE_BYTES];
    float act[ACT_FLOATS];            // GEMV activations; attention scratch
    float kv[2][ATT_TILE][HD];        // attention K / V tile
    float xs[RMAX][XS_MAX];           // this CTA's rows of the residual stream
    float part[MAX_PARTS * RMAX];     // GEMV partial sums of the slice
    int slice[M_FIXED][2];            // rows [r0, r1) of each fixed matrix owned by this CTA
    float red[NWARPS * RMAX];
    float inv[RMAX];                  // 1/rms of the staged rows, for the GEMV epilogue
    unsigned long long keys[NWARPS];
    uint64_t full[NSTAGES];
    uint64_t empty[NSTAGES];
    uint64_t kvbar;
    int abort_flag;
    int issued;     // chunks the producer has issued
    int bcast;
    int kv_rows;    // cached rows of the prefetched tile (0: nothing in flight)
    int barflag[3];     // OR reductions of the compute-warp barrier, rotating
};

// CTA-level barriers of the compute warps: Compute::cta_sync / cta_or
#define named_sync() cta_sync()
#define named_or(v) cta_or(v)

// ------------------------------------------------------------------ program walk

__device__ __forceinline__ int mat_rows(Mat m, int head_rows) {
    switch (m) {
        case M_QKV: return QKV_ROWS;
        case M_O: return H;
        case M_OH: return HKV * H;  // by kv head
        case M_GU: return GU_ROWS;
        case M_D: return H;
        default: return head_rows;
    }
}
__device__ __forceinline__ int mat_k(Mat m) {
    switch (m) {
        case M_O: return QDIM;
        case M_OH: return KO;
        case M_D: return INTER;
        default: return H;
    }
}
// rows [r0, r1) of an N-row matrix owned by CTA b of G (pairs for gate/up;
// QKV and the O projection by kv head: rows of the head's block split over
// the CTAs of its group)
__device__ __forceinline__ void mat_slice(Mat m, int n, int b, int g, int &r0, int &r1) {
    if (m == M_QKV || m == M_OH) {
        int h, j, nj;
        head_group(b, g, h, j, nj);
        const int per = n / HKV;
        r0 = h * per + j * per / nj;
        r1 = h * per + (j + 1) * per / nj;
    } else if (m == M_GU) {
        int p = n / 2;
        r0 = 2 * static_cast<int>(static_cast<long long>(b) * p / g);
        r1 = 2 * static_cast<int>(static_cast<long long>(b + 1) * p / g);
    } else {
        r0 = static_cast<int>(static_cast<long long>(b) * n / g);
        r1 = static_cast<int>(static_cast<long long>(b + 1) * n / g);
    }
}
__device__ __forceinline__ int stage_rows(int wdt, int k, Mat m) {
    int r = STAGE_BYTES / row_bytes(wdt, k);
    return m == M_GU ? (r & ~1) : r;  // even for gate/up: a SwiGLU pair never straddles two stages
}

// ------------------------------------------------------------------ producer

template <int WDT>
struct Producer {
    Smem *sm;
    int seq = 0;  // chunks issued
    bool ok = true;
    __device__ void matrix(const uint8_t *w, Mat m, int head_rows, bool keep) {
        if (!ok) return;
        int n = mat_rows(m, head_rows), k = mat_k(m), rb = row_bytes(WDT, k);
        int r0, r1;
        mat_slice(m, n, blockIdx.x, gridDim.x, r0, r1);
        int sr = stage_rows(WDT, k, m);
        uint64_t pol = l2_policy(keep);
        for (int r = r0; r < r1; r += sr) {
            int nr = min(sr, r1 - r);
            int slot = seq % NSTAGES;
            if (seq >= NSTAGES) {
                uint32_t par = ((seq / NSTAGES) - 1) & 1;
                if (!mbar_wait(&sm->empty[slot], par, &sm->abort_flag)) {
                    ok = false;
                    return;
                }
            }
            uint32_t bytes = static_cast<uint32_t>(nr * rb);
            mbar_arrive_tx(&sm->full[slot], bytes);
            bulk_g2s(sm->ring[slot], w + static_cast<size_t>(r) * rb, bytes, &sm->full[slot], pol);
            ++seq;
            sm->issued = seq;
        }
    }

};

// ------------------------------------------------------------------ compute

// the draw of a frame's code from the logits lg[V] of the last head (NCT
// threads; talker: ChooseCode0's processors first, as choose0_value)
static_assert(sizeof(SampleScratch) <= sizeof(float) * ACT_FLOATS, "the draw's scratch lives in the activation buffer");

__device__ __noinline__ int frame_draw(const float *lg, int V, SampleParams p, float u, SampleScratch *ss, int tid,
                                       bool talker, int vocab, int eos, int hist_now, const unsigned char *seen,
                                       float penalty) {
    if (talker)
        return sample_draw<NCT>(
            [&](int i) {
                const float s = __ldcg(lg + i);
                if (i >= vocab - 1024 && i != eos) return -INFINITY;
                if (i == eos && hist_now < 2) return -INFINITY;
                if (penalty != 1.0f && seen[i]) return s > 0.f ? __fdiv_rn(s, penalty) : s * penalty;
                return s;
            },
            V, p, u, ss, tid);
    return sample_draw<NCT>([&](int i) { return __ldcg(lg + i); }, V, p, u, ss, tid);
}

// KV16: the K/V cache holds half floats (a compile-time choice: a runtime
// flag in the attention loop slowed the float32 frame by ~15 %)
template <int WDT, int KV16>
struct Compute {
    Smem *sm;
    const Job *job;
    int seq = 0;          // chunks consumed
    unsigned target = 0;  // grid barrier target
    bool ok = true;
    int hist_now = 0;     // history length for ChooseCode0 (frame mode)
    uint32_t kv_phase = 0;
    int tid, warp, lane;
    int c0, c1;           // this CTA's residual rows

    int barc = 0;         // cta_or calls so far (the same count in every thread)

    // Barrier of the compute warps (hardware barrier 1, 480 threads), each
    // warp converged first.  With pred: also ORs pred over the compute
    // threads through a rotating shared flag (no bar.red).
    __device__ __forceinline__ void cta_sync() {
        __syncwarp();
        asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
    }
    __device__ __forceinline__ bool cta_or(bool pred) {
        __syncwarp();
        const bool wp = __any_sync(0xffffffffu, pred);
        const int k = barc++;
        if (lane == 0 && wp) sm->barflag[k % 3] = 1;
        asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory");
        const bool r = *reinterpret_cast<volatile int *>(&sm->barflag[k % 3]) != 0;
        // the flag of call k+2 was last read at call k-1: free to clear
        if (tid == 0) sm->barflag[(k + 2) % 3] = 0;
        return r;
    }

    int ntrace = 0;
    __device__ __forceinline__ void mark(int tag) {
        if (job->trace && blockIdx.x == 0 && tid == 0 && ntrace < job->trace_cap)
            job->trace[ntrace++] = (static_cast<unsigned long long>(tag) << 48) | (gtimer() & 0xFFFFFFFFFFFFull);
    }

    __device__ void fail(int code, int where) {
        if (ok) {
            ok = false;
            atomicCAS(job->s.err, 0, code);
            atomicCAS(job->s.err + 1, 0, where);
            sm->abort_flag = 1;
        }
    }

    // ---------------------------------------------------------------- tagged handoffs

    // The QKV rows (to the attention) and the residual stream after the down
    // projection (to the next layer's staging) pass between CTAs as tagged
    // words instead of through a grid barrier: the producer stores value and
    // tag in one 8-byte word, the consumer re-reads until the word carries
    // the tag of this handoff.  Every CTA draws the tags in the same order.
    unsigned hseq = 0;                     // handoffs so far in this launch
    unsigned cur_tag = 0;                  // the tag the next tagged epilogue stores
    unsigned long long *x8out = nullptr;   // E_RESID: also store the rows tagged here
    unsigned key_tag = 0;                  // E_HEAD*: store the CTA's argmax key tagged (0: plain)
    const float *next_rows = nullptr;      // E_HEAD*: the table whose row the winning index selects next
    __device__ __forceinline__ unsigned next_tag() {
        ++hseq;
        return (job->epoch << TAG_SEQ_BITS) | (hseq & ((1u << TAG_SEQ_BITS) - 1u));
    }
    // 4 consecutive tagged words (16-byte aligned) once all carry `tag`;
    // bounded like the barriers (false: timeout or another CTA's failure)
    __device__ __forceinline__ bool poll4(const unsigned long long *p, unsigned tag, float4 &out) {
        unsigned long long a, b, c, d;
        ld_tagged2(p, a, b);
        ld_tagged2(p + 2, c, d);
        if (!(tag_is(a, tag) && tag_is(b, tag) && tag_is(c, tag) && tag_is(d, tag))) {
            const long long t0 = clock64();
            while (true) {
                if (!(tag_is(a, tag) && tag_is(b, tag))) ld_tagged2(p, a, b);
                if (!(tag_is(c, tag) && tag_is(d, tag))) ld_tagged2(p + 2, c, d);
                if (tag_is(a, tag) && tag_is(b, tag) && tag_is(c, tag) && tag_is(d, tag)) break;
                if (*reinterpret_cast<volatile int *>(job->s.err) != 0 || clock64() - t0 > job->wait_cycles)
                    return false;
            }
        }
        out = make_float4(__uint_as_float(static_cast<unsigned>(a)), __uint_as_float(static_cast<unsigned>(b)),
                          __uint_as_float(static_cast<unsigned>(c)), __uint_as_float(static_cast<unsigned>(d)));
        return true;
    }

    // grid-wide barrier among the compute warps of all CTAs: release-add on
    // a monotonic counter, acquire-poll until every CTA has arrived.  It also
    // makes `ok` uniform over the CTA (any thread's failure fails all).
    __device__ void grid_sync(int where) {
        const bool bad = named_or(!ok);
        mark(100 + where);  // arrival of CTA 0
        if (tid == 0) {
            target += gridDim.x;
            int b = bad ? 1 : 0;
            if (!bad) {
                unsigned *bar = job->s.bar;
                asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
                const long long t0 = clock64();
                const unsigned want = target + static_cast<unsigned>(job->bar_extra);
                while (true) {
                    unsigned v;
                    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
                    if (v >= want) break;
                    if (*reinterpret_cast<volatile int *>(job->s.err) != 0) {
                        fail(ERR_TIMEOUT, where);
                        b = 1;
                        break;
                    }
                    if (clock64() - t0 > job->wait_cycles) {
                        fail(ERR_TIMEOUT, where);
                        b = 1;
                        break;
                    }
                }
            }
            sm->bcast = b;
        }
        named_sync();
        ok = sm->bcast == 0;
        mark(200 + where);  // departure
    }

    // ---------------------------------------------------------------- staging

    // act[r][0..H) = x_r * w for the rows x_r = ((a + b) + c) (up to 3
    // addends: the summation order of TQwenTalker.NextFrame), and the sums
    // of squares of x_r per warp in red[]: the RMSNorm scale 1/rms(x_r) is
    // applied by the GEMV epilogue (norm_inv), so staging needs one barrier.
    // With init_resid, this CTA's residual rows [c0, c1) come from the sum.
    //  opart != NULL (per-head path): the rows are a[r] (+ b[r] + c[r]) plus
    //  the O projection, the sum of its HKV per-kv-head partials
    //  opart[r][h][..] in head order.
    //  a8 != NULL: the rows a[r] are the tagged words a8[r][..] of handoff
    //  a8tag instead (the residual stream as the down projection left it).
    __device__ void stage_norm(const float *const *a, const float *const *b, const float *const *c, int R,
                               const float *w, bool init_resid, const float *opart = nullptr,
                               const unsigned long long *a8 = nullptr, unsigned a8tag = 0) {
        float ss[RMAX] = {0.f, 0.f, 0.f, 0.f};
        for (int idx = tid; idx < R * (H / 4); idx += NCT) {
            const int r = idx / (H / 4), i = 4 * (idx - r * (H / 4));
            float4 v;
            if (a8) {
                // warp-uniform verdict (every lane of a warp runs the same iterations)
                if (!__all_sync(0xffffffffu, poll4(a8 + r * H + i, a8tag, v))) fail(ERR_TIMEOUT, 60);
            } else {
                v = ldcg4(a[r] + i);
            }
            float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
            if (opart) {
                // all HKV loads in flight together, summed in head order
                const float *op = opart + static_cast<size_t>(r) * (HKV * H) + i;
                float4 t[HKV];
#pragma unroll
                for (int hh = 0; hh < HKV; ++hh) t[hh] = ldcg4(op + hh * H);
                y = t[0];
#pragma unroll
                for (int hh = 1; hh < HKV; ++hh) {
                    y.x = y.x + t[hh].x; y.y = y.y + t[hh].y; y.z = y.z + t[hh].z; y.w = y.w + t[hh].w;
                }
            }
            if (b && b[r]) {
                const float4 t = ldcg4(b[r] + i);
                v.x = v.x + t.x; v.y = v.y + t.y; v.z = v.z + t.z; v.w = v.w + t.w;
            }
            if (c && c[r]) {
                const float4 t = ldcg4(c[r] + i);
                v.x = v.x + t.x; v.y = v.y + t.y; v.z = v.z + t.z; v.w = v.w + t.w;
            }
            if (opart) {
                v.x = v.x + y.x; v.y = v.y + y.y; v.z = v.z + y.z; v.w = v.w + y.w;
            }
            const float4 g = *reinterpret_cast<const float4 *>(w + i);
            *reinterpret_cast<float4 *>(sm->act + r * H + i) = make_float4(v.x * g.x, v.y * g.y, v.z * g.z, v.w * g.w);
            float s = v.x * v.x;
            s = fmaf(v.y, v.y, s);
            s = fmaf(v.z, v.z, s);
            s = fmaf(v.w, v.w, s);
#pragma unroll
            for (int rr = 0; rr < RMAX; ++rr)
                if (rr == r) ss[rr] += s;
            if (init_resid) {
                const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (i + j >= c0 && i + j < c1) sm->xs[r][i + j - c0] = vv[j];
            }
        }
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
            if (r < R) {
                const float t = warp_sum(ss[r]);
                if (lane == 0) sm->red[warp * RMAX + r] = t;
            }
        }
        named_sync();
    }
    // 1/rms of staged row r (after stage_norm's barrier)
    __device__ __forceinline__ float norm_inv(int r, float eps) const {
        float t = 0.f;
        for (int w2 = 0; w2 < NCW; ++w2) t += sm->red[w2 * RMAX + r];
        return 1.0f / sqrtf(t / static_cast<float>(H) + eps);
    }

    __device__ void stage_copy(const float *src, int R, int k) {
        for (int i = tid; i < R * k / 4; i += NCT)
            reinterpret_cast<float4 *>(sm->act)[i] = ldcg4(src + 4 * i);
        named_sync();
    }

    // the attention output of all 16 query heads: combine the S partials of
    // each (row, head): o = sum_s o_s e^(m_s - M) / sum_s l_s e^(m_s - M).
    // A warp per (row, head): lane s brings (m_s, l_s) (S <= 32), lane d
    // dims 4d..4d+3 of 4 splits per round trip.
    __device__ __forceinline__ void stage_attn(int R, int S) {
        const size_t split_stride = static_cast<size_t>(RMAX) * 2 * PSTRIDE;
        for (int task = warp; task < R * HQ; task += NCW) {
            const int r = task / HQ, qh = task - r * HQ;
            const int h = qh >> 1, q = qh & 1;
            const float *base = job->s.part + ((static_cast<size_t>(h) * S * RMAX + r) * 2 + q) * PSTRIDE;
            float ms = -INFINITY, ls = 0.f;
            if (lane < S) {
                const float2 u = __ldcg(reinterpret_cast<const float2 *>(base + lane * split_stride + HD));
                ms = u.x;
                ls = u.y;
            }
            // the first splits' partial outputs travel with the (max, sum) loads
            constexpr int PRE = WDT == WDT_Q8 ? 4 : 1;  // float32 weights leave fewer registers
            float4 op[PRE];
#pragma unroll
            for (int j = 0; j < PRE; ++j)
                if (j < S) op[j] = ldcg4(base + j * split_stride + 4 * lane);
            float M = ms;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            const float e = ms == -INFINITY ? 0.f : expf(ms - M);
            const float L = warp_sum(ls * e);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < PRE; ++j) {
                const float es = __shfl_sync(0xffffffffu, e, j);
                if (j < S) {
                    acc.x = fmaf(op[j].x, es, acc.x);
                    acc.y = fmaf(op[j].y, es, acc.y);
                    acc.z = fmaf(op[j].z, es, acc.z);
                    acc.w = fmaf(op[j].w, es, acc.w);
                }
            }
            for (int s0 = PRE; s0 < S; s0 += 4) {
                float4 o[4];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (s0 + j < S) o[j] = ldcg4(base + (s0 + j) * split_stride + 4 * lane);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float es = __shfl_sync(0xffffffffu, e, (s0 + j) & 31);
                    if (s0 + j < S) {
                        acc.x = fmaf(o[j].x, es, acc.x);
                        acc.y = fmaf(o[j].y, es, acc.y);
                        acc.z = fmaf(o[j].z, es, acc.z);
                        acc.w = fmaf(o[j].w, es, acc.w);
                    }
                }
            }
            const float inv = 1.0f / L;
            *reinterpret_cast<float4 *>(sm->act + r * QDIM + qh * HD + 4 * lane) =
                make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
        named_sync();
    }

    // ---------------------------------------------------------------- GEMV

    // Epilogue kinds
    enum Epi { E_STORE, E_RESID, E_SWIGLU, E_HEAD, E_HEAD0, E_TAGGED };

    // rows [r0, r1) of matrix m owned by this CTA (the fixed matrices from
    // the table filled at the start of the launch)
    __device__ __forceinline__ void slice_of(Mat m, int head_rows, int &r0, int &r1) const {
        if (m < M_FIXED) {
            r0 = sm->slice[m][0];
            r1 = sm->slice[m][1];
        } else {
            mat_slice(m, head_rows, blockIdx.x, gridDim.x, r0, r1);
        }
    }

    // GEMV over this CTA's slice of matrix m; activations staged in sm->act
    // as [R][K].  Work items are (row pair, 1024-wide K segment), the
    // activations loaded once for both rows, numbered over the whole slice
    // chunk by chunk; warp w takes items w, w+15, ...  Each warp waits for
    // the stages it reads and releases every stage of the phase itself (the
    // empty barriers count the 15 compute warps), so the phase has a single
    // CTA barrier, before the epilogue.  eps >= 0: the rows were staged by
    // stage_norm and y is scaled by their 1/rms.
    //  E_STORE: out[r*ld + row] = y
    //  E_TAGGED: the same as a tagged word (out is the 64-bit word array),
    //  tag cur_tag
    //  E_RESID: residual row: xs[r][row-c0] += y, out[r*H + row] = xs (and,
    //  with x8out, the same as a tagged word of x8out, tag cur_tag)
    //  E_SWIGLU: out[r*ld + row/2] = silu(y_gate) * y_up
    //  E_HEAD / E_HEAD0: out[row] = y (R == 1), the CTA's argmax key to
    //  job->s.arg; E_HEAD0 applies ChooseCode0's processors first.
    //  RR: activation rows the dot-product loop is compiled for (1, or RMAX
    //  with the rows past R skipped): gemv() dispatches on R.
    template <int K>
    __device__ __forceinline__ void gemv(Mat m, int head_rows, int R, int kind, float *out, int ld, float eps) {
        if (R == 1)
            gemv_rr<K, 1>(m, head_rows, R, kind, out, ld, eps);
        else
            gemv_rr<K, RMAX>(m, head_rows, R, kind, out, ld, eps);
    }
    template <int K, int RR>
    __device__ __forceinline__ void gemv_rr(Mat m, int head_rows, int R, int kind, float *out, int ld, float eps) {
        constexpr int SEGW = K < 1024 ? K : 1024;  // K segment of one item
        constexpr int SEG = K / SEGW;
        const int rb = row_bytes(WDT, K);
        int r0, r1;
        slice_of(m, head_rows, r0, r1);
        const int nrows = r1 - r0;
        const int sr = stage_rows(WDT, K, m);
        const int nchunks = (nrows + sr - 1) / sr;
        const int pairs_full = (sr + 1) >> 1;  // pairs of a full chunk
        int it = warp;                         // next item of this warp
        bool good = __all_sync(0xffffffffu, ok);  // warp-uniform (the stage waits use warp votes)
        // the staged rows' 1/rms, once (the barrier before the epilogue
        // publishes it): the last warp has the fewest items
        if (eps >= 0.f && warp == NCW - 1 && lane < R) sm->inv[lane] = norm_inv(lane, eps);
        for (int ch = 0; ch < nchunks; ++ch) {
            const int slot = (seq + ch) % NSTAGES;
            const uint32_t par = ((seq + ch) / NSTAGES) & 1;
            const int nr = min(sr, nrows - ch * sr);
            const int item_end = (ch * pairs_full + ((nr + 1) >> 1)) * SEG;  // items of chunks <= ch
            // every warp observes every stage (so that no parity is skipped)
            // before it releases it; warp-uniform verdict for the shuffles
            if (good) {
                const bool got = __all_sync(0xffffffffu, mbar_wait(&sm->full[slot], par, &sm->abort_flag));
                if (!got) {
                    good = false;
                    fail(ERR_TIMEOUT, 100 + m);
                }
            }
            const uint8_t *base = sm->ring[slot];
            for (; it < item_end; it += NCW) {
                if (!good) continue;
                const int pair = it / SEG - ch * pairs_full, seg = it % SEG;
                const int ra = 2 * pair;
                const bool two = ra + 1 < nr;
                const uint8_t *rowa = base + ra * rb;
                const uint8_t *rowb = two ? rowa + rb : rowa;
                float aa[RR], ab[RR];
#pragma unroll
                for (int r = 0; r < RR; ++r) aa[r] = ab[r] = 0.f;
#pragma unroll
                    for (int g = 0; g < SEGW / 128; ++g) {
                        const int e = seg * SEGW + 128 * g + 4 * lane;  // first of this lane's 4 elements
                        float4 wa, wb;
                        float da = 1.f, db = 1.f;
                        if (WDT == WDT_Q8) {
                            wa = dq4(*reinterpret_cast<const uint32_t *>(rowa + e));
                            wb = dq4(*reinterpret_cast<const uint32_t *>(rowb + e));
                            da = __half2float(reinterpret_cast<const __half *>(rowa + K)[e >> 5]);
                            db = __half2float(reinterpret_cast<const __half *>(rowb + K)[e >> 5]);
                        } else {
                            wa = *reinterpret_cast<const float4 *>(rowa + 4 * e);
                            wb = *reinterpret_cast<const float4 *>(rowb + 4 * e);
                        }
#pragma unroll
                        for (int r = 0; r < RR; ++r) {
                            if (RR == 1 || r < R) {
                                const float4 xv = *reinterpret_cast<const float4 *>(sm->act + r * K + e);
                                float pa = wa.x * xv.x, pb = wb.x * xv.x;
                                pa = fmaf(wa.y, xv.y, pa);
                                pb = fmaf(wb.y, xv.y, pb);
                                pa = fmaf(wa.z, xv.z, pa);
                                pb = fmaf(wb.z, xv.z, pb);
                                pa = fmaf(wa.w, xv.w, pa);
                                pb = fmaf(wb.w, xv.w, pb);
                                if (WDT == WDT_Q8) {
                                    aa[r] = fmaf(da, pa, aa[r]);
                                    ab[r] = fmaf(db, pb, ab[r]);
                                } else {
                                    aa[r] += pa;
                                    ab[r] += pb;
                                }
                            }
                        }
                    }
                const int row = ch * sr + ra;  // row within the slice
#pragma unroll
                for (int r = 0; r < RR; ++r) {
                    if (RR == 1 || r < R) {
                        const float s = warp_sum2(aa[r], ab[r], lane);
                        if (lane == 0) sm->part[(row * SEG + seg) * RMAX + r] = s;
                        if (lane == 16 && two) sm->part[((row + 1) * SEG + seg) * RMAX + r] = s;
                    }
                }
            }
            // this warp is done with the stage
            __syncwarp();
            if (lane == 0 && good) mbar_arrive(&sm->empty[slot]);
        }
        seq += nchunks;
        named_sync();
        if (*reinterpret_cast<volatile int *>(&sm->abort_flag)) {
            ok = false;
            return;
        }
        // epilogue over the slice
        unsigned long long best = 0ull;
        if (kind == E_SWIGLU) {
            const int np = nrows / 2;
            for (int idx = tid; idx < np * R; idx += NCT) {
                const int p = idx / R, r = idx - p * R;
                float g = 0.f, v = 0.f;
#pragma unroll
                for (int sg = 0; sg < SEG; ++sg) {
                    g += sm->part[((2 * p) * SEG + sg) * RMAX + r];
                    v += sm->part[((2 * p + 1) * SEG + sg) * RMAX + r];
                }
                if (eps >= 0.f) {
                    const float inv = sm->inv[r];
                    g *= inv;
                    v *= inv;
                }
                const float s = g / (1.0f + expf(-g));
                out[r * ld + (r0 + 2 * p) / 2] = s * v;
            }
        } else {
            for (int idx = tid; idx < nrows * R; idx += NCT) {
                const int row = idx / R, r = idx - row * R;
                float y = 0.f;
#pragma unroll
                for (int sg = 0; sg < SEG; ++sg) y += sm->part[(row * SEG + sg) * RMAX + r];
                if (eps >= 0.f) y *= sm->inv[r];
                const int orow = r0 + row;
                if (kind == E_STORE) {
                    out[r * ld + orow] = y;
                } else if (kind == E_TAGGED) {
                    st_tagged(reinterpret_cast<unsigned long long *>(out) + r * ld + orow, y, cur_tag);
                } else if (kind == E_RESID) {
                    const float v = sm->xs[r][orow - c0] + y;
                    sm->xs[r][orow - c0] = v;
                    out[r * H + orow] = v;
                    if (x8out) st_tagged(x8out + r * H + orow, v, cur_tag);
                } else {
                    out[orow] = y;
                    const float w = kind == E_HEAD0 ? choose0_value(orow, y) : y;
                    const unsigned long long k = argkey(w, orow);
                    best = k > best ? k : best;
                }
            }
        }
        if (kind == E_HEAD || kind == E_HEAD0) {
            // CTA-wide max of the keys
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
                best = t > best ? t : best;
            }
            if (lane == 0) sm->keys[warp] = best;
            named_sync();
            if (warp == 0) {
                unsigned long long b = lane < NCW ? sm->keys[lane] : 0ull;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
                    b = t > b ? t : b;
                }
                if (key_tag) {
                    // tagged key: the float bits, the tag, the index (< 4096)
                    const unsigned idx = static_cast<unsigned>(key_index(b)) & 0xFFFu;
                    const unsigned long long kt = (b & 0xFFFFFFFF00000000ull) |
                                                  (static_cast<unsigned long long>(key_tag & 0xFFFFFu) << 12) |
                                                  (0xFFFu - idx);
                    if (lane == 0)
                        asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(job->s.arg + blockIdx.x), "l"(kt)
                                     : "memory");
                } else if (lane == 0) {
                    job->s.arg[blockIdx.x] = b;
                }
                // the row the next step gathers if this CTA's candidate wins,
                // brought into L2 while the keys meet
                if (next_rows && b != 0ull) {
                    const char *row = reinterpret_cast<const char *>(next_rows + static_cast<size_t>(key_index(b)) * H);
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(row + 128 * lane));
                }
            }
        }
    }

    // TQwenTalker.ChooseCode0 (talker.pas:595-630), greedy, for one logit:
    // the last 1024 ids forbidden but eos, eos forbidden before 2 frames,
    // repetition penalty once per distinct code already returned
    __device__ __forceinline__ float choose0_value(int i, float s) {
        const int vocab = job->tvocab;
        if (i >= vocab - 1024 && i != job->eos) return -INFINITY;
        if (i == job->eos && hist_now < 2) return -INFINITY;
        if (job->penalty != 1.0f && job->seen[i]) return s > 0.f ? __fdiv_rn(s, job->penalty) : s * job->penalty;
        return s;
    }

    // after a grid barrier: the code drawn from the logits of the last head
    // (every compute thread of the CTA calls it; sm->act is the scratch);
    // code 0 (talker) from the values after ChooseCode0's processors.  The
    // draw is a call (frame_draw), so that the layer code stays compact.
    __device__ __forceinline__ int sample_code(int V, const SampleParams &p, float u, bool talker) {
        return frame_draw(job->s.logits, V, p, u, reinterpret_cast<SampleScratch *>(sm->act), tid, talker,
                          job->tvocab, job->eos, hist_now, job->seen, job->penalty);
    }

    // the winning index over all CTAs' tagged keys of handoff tag (no
    // barrier): warp 0 polls the keys and reduces, the CTA reads its verdict;
    // ok is uniform over the CTA afterwards
    __device__ int reduce_argmax_tagged(unsigned tag) {
        if (warp == 0) {
            unsigned long long b = 0ull;
            bool got = true;
            for (int i = lane; i < static_cast<int>(gridDim.x); i += 32) {
                const unsigned long long *p = job->s.arg + i;
                unsigned long long k;
                const long long t0 = clock64();
                while (true) {
                    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(k) : "l"(p) : "memory");
                    if (static_cast<unsigned>((k >> 12) & 0xFFFFFu) == (tag & 0xFFFFFu)) break;
                    if (*reinterpret_cast<volatile int *>(job->s.err) != 0 || clock64() - t0 > job->wait_cycles) {
                        got = false;
                        break;
                    }
                }
                if (!got) break;
                b = k > b ? k : b;
            }
            got = __all_sync(0xffffffffu, got);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
                b = t > b ? t : b;
            }
            if (!got) fail(ERR_TIMEOUT, 62);
            if (lane == 0) sm->bcast = static_cast<int>(0xFFFu - static_cast<unsigned>(b & 0xFFFu));
        }
        named_sync();
        if (*reinterpret_cast<volatile int *>(&sm->abort_flag)) ok = false;
        const int code = sm->bcast;
        named_sync();  // sm->bcast is the grid barrier's word too
        return code;
    }

    // after a grid barrier: the winning index over all CTAs' keys
    __device__ int reduce_argmax() {
        unsigned long long b = 0ull;
        for (int i = lane; i < static_cast<int>(gridDim.x); i += 32) {
            const unsigned long long k = __ldcg(job->s.arg + i);
            b = k > b ? k : b;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
            b = t > b ? t : b;
        }
        return key_index(b);
    }

    // ---------------------------------------------------------------- attention

    // The attention item of this CTA for a context of T positions: kv head
    // h, split s over positions [p0, p1); false when the CTA has none.
    __device__ __forceinline__ bool att_item(int T, int &S, int &h, int &s, int &p0, int &p1) {
        S = att_splits(T, gridDim.x);
        const int C = (T + S - 1) / S;
        const int item = blockIdx.x;
        if (item >= HKV * S) return false;
        h = item / S;
        s = item - h * S;
        p0 = s * C;
        p1 = min(T, p0 + C);
        return true;
    }

    // Issued at the end of P1, before the barrier: the cached K/V rows of the
    // first tile of this CTA's split (positions < L0, written in earlier
    // steps), bulk-copied into sm->kv.  Thread 0.
    __device__ void prefetch_kv(const DCtx &kv, int layer, int R, int L0, bool head_path) {
        if (tid == 0) {
            sm->kv_rows = 0;
            int S, h, s, p0, p1;
            bool have = false;
            if (head_path) {
                int j, nj;
                head_group(blockIdx.x, gridDim.x, h, j, nj);
                p0 = 0;
                p1 = L0 + R;
                have = true;
            } else {
                have = att_item(L0 + R, S, h, s, p0, p1);
            }
            if (ok && have) {
                const int n = min(min(p1, L0), p0 + ATT_TILE) - p0;
                if (n > 0) {
                    constexpr int es = KV16 ? 2 : 4;
                    const size_t off = ((static_cast<size_t>(layer) * HKV + h) * kv.max_pos + p0) * HD * es;
                    // the rows were written through the generic proxy
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    mbar_arrive_tx(&sm->kvbar, static_cast<uint32_t>(2 * n * HD * es));
                    bulk_g2s(&sm->kv[0][0][0], static_cast<const char *>(kv.k) + off, static_cast<uint32_t>(n * HD * es),
                             &sm->kvbar);
                    bulk_g2s(&sm->kv[1][0][0], static_cast<const char *>(kv.v) + off, static_cast<uint32_t>(n * HD * es),
                             &sm->kvbar);
                    sm->kv_rows = n;
                }
            }
        }
    }

    // P2 for this CTA's item: q (heads 2h, 2h+1) / k / v of the new rows
    // normed and rotated, the new K/V appended to the cache (split 0), then
    // online-softmax attention over [p0, p1) with positions spread over the
    // warps; the partial (o, max, sum) of every (row, q head) to global.
    //  head_path (a context of one tile): CTA b takes its group's kv head and
    //  the whole context, CTA 0 of the group appends, and the normalised
    //  output of row r goes to act[r][KO] for the O projection by head.
    //  The new rows arrive as the tagged words of handoff qtag (the QKV
    //  GEMV's epilogue): each lane polls its 4 values.
    __device__ void attention(const DLayer &Ly, const DCtx &kv, int layer, int R, int L0, float eps,
                              bool head_path, unsigned qtag) {
        const int T = L0 + R;
        int S, h, s, p0, p1;
        bool append;
        if (head_path) {
            int j, nj;
            head_group(blockIdx.x, gridDim.x, h, j, nj);
            S = 1;
            s = 0;
            p0 = 0;
            p1 = T;
            append = j == 0;
        } else {
            if (!att_item(T, S, h, s, p0, p1)) return;
            append = s == 0;
        }
        const bool prefetched = sm->kv_rows > 0;
        // shared layout inside sm->act: [head path: o[R][KO]] | q[R][2][HD] | kn[R][HD] | vn[R][HD] | warp states
        float *qs = sm->act + (head_path ? RMAX * KO : 0);
        float *kn = qs + RMAX * 2 * HD;
        float *vn = kn + RMAX * HD;
        float *wst = vn + RMAX * HD;  // [NCW][PSTRIDE]
        const int half = HD / 2;
        // 1. the new rows
        for (int vec = warp; vec < 4 * R; vec += NCW) {
            const int r = vec >> 2, t = vec & 3;  // t: 0,1 = q heads, 2 = k, 3 = v
            // QKV rows by kv head: q(2h), q(2h+1), k(h), v(h)
            const unsigned long long *src = job->s.qkv + r * QKV_ROWS + h * QKV_HEAD + t * HD;
            // the norm weights and the RoPE row do not depend on the rows:
            // their loads go out together with the row's
            float4 g = make_float4(0.f, 0.f, 0.f, 0.f), cs = g, sn = g;
            if (t < 3) {
                const float *nw = t < 2 ? Ly.q_norm : Ly.k_norm;
                const int e0 = (4 * lane) & (half - 1);
                const size_t ro = static_cast<size_t>(L0 + r) * half + e0;
                g = *reinterpret_cast<const float4 *>(nw + 4 * lane);
                cs = *reinterpret_cast<const float4 *>(job->rope_cos + ro);
                sn = *reinterpret_cast<const float4 *>(job->rope_sin + ro);
            }
            float4 x;
            if (!__all_sync(0xffffffffu, poll4(src + 4 * lane, qtag, x))) fail(ERR_TIMEOUT, 41);
            float y[4] = {x.x, x.y, x.z, x.w};
            if (t < 3) {
                const float ss = warp_sum(y[0] * y[0] + y[1] * y[1] + y[2] * y[2] + y[3] * y[3]);
                const float inv = 1.0f / sqrtf(ss / static_cast<float>(HD) + eps);
                y[0] = g.x * (y[0] * inv);
                y[1] = g.y * (y[1] * inv);
                y[2] = g.z * (y[2] * inv);
                y[3] = g.w * (y[3] * inv);
                const float cv[4] = {cs.x, cs.y, cs.z, cs.w}, sv[4] = {sn.x, sn.y, sn.z, sn.w};
                float o[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float partner = __shfl_xor_sync(0xffffffffu, y[j], 16);
                    o[j] = lane < 16 ? y[j] * cv[j] - partner * sv[j] : y[j] * cv[j] + partner * sv[j];
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) y[j] = o[j];
            }
            if (KV16 && t >= 2) {
                // a half-float cache: this step reads the new K/V as later
                // steps will, rounded to fp16
#pragma unroll
                for (int j = 0; j < 4; ++j) y[j] = __half2float(__float2half_rn(y[j]));
            }
            float *dst = t < 2 ? qs + (r * 2 + t) * HD : (t == 2 ? kn + r * HD : vn + r * HD);
            *reinterpret_cast<float4 *>(dst + 4 * lane) = make_float4(y[0], y[1], y[2], y[3]);
            if (append && t >= 2) {
                const size_t e = ((static_cast<size_t>(layer) * HKV + h) * kv.max_pos + (L0 + r)) * HD + 4 * lane;
                void *cache = t == 2 ? kv.k : kv.v;
                if (KV16) {
                    __half2 hh[2] = {__floats2half2_rn(y[0], y[1]), __floats2half2_rn(y[2], y[3])};
                    *reinterpret_cast<uint2 *>(static_cast<__half *>(cache) + e) = *reinterpret_cast<uint2 *>(hh);
                } else {
                    *reinterpret_cast<float4 *>(static_cast<float *>(cache) + e) = make_float4(y[0], y[1], y[2], y[3]);
                }
            }
        }
        bool landed = true;
        if (prefetched) {
            // every thread waits for the tile (bounded); a wait that gave up
            // leaves sm->kv_rows set and the phase unchanged, so that the
            // exit drains the copy
            landed = mbar_wait(&sm->kvbar, kv_phase, &sm->abort_flag);
            if (landed)
                kv_phase ^= 1u;
            else
                fail(ERR_TIMEOUT, 40);
        }
        named_sync();
        if (tid == 0 && landed) sm->kv_rows = 0;
        // 2. online softmax: warps grouped by (row, q head), positions strided
        const float scale = 1.0f / sqrtf(static_cast<float>(HD));
        const int nc = 2 * R, npw = NCW / nc;
        const int combo = warp / npw, sub = warp - combo * npw;
        const bool active = combo < nc;
        const int cr = combo >> 1, cq = combo & 1;
        float m = -INFINITY, l = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
        const size_t hoff = (static_cast<size_t>(layer) * HKV + h) * kv.max_pos * HD;
        // a half-float cache keeps its tiles in shared memory as [ATT_TILE][HD] halves
        const __half *ktile16 = reinterpret_cast<const __half *>(&sm->kv[0][0][0]);
        const __half *vtile16 = reinterpret_cast<const __half *>(&sm->kv[1][0][0]);
        float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
        if (active) q = *reinterpret_cast<const float4 *>(qs + (cr * 2 + cq) * HD + 4 * lane);
        for (int tp = p0; tp < p1; tp += ATT_TILE) {
            const int nt = min(ATT_TILE, p1 - tp);
            const int cached = max(0, min(nt, L0 - tp));
            if (tp != p0 || !prefetched) {
                // a tile that was not prefetched: plain loads of its cached rows
                if (tp != p0) named_sync();
                if (KV16) {
                    const __half *kb = static_cast<const __half *>(kv.k) + hoff, *vb = static_cast<const __half *>(kv.v) + hoff;
                    for (int i = tid; i < cached * (HD / 8); i += NCT) {
                        const size_t g = static_cast<size_t>(tp) * HD + 8 * static_cast<size_t>(i);
                        reinterpret_cast<uint4 *>(&sm->kv[0][0][0])[i] = __ldcg(reinterpret_cast<const uint4 *>(kb + g));
                        reinterpret_cast<uint4 *>(&sm->kv[1][0][0])[i] = __ldcg(reinterpret_cast<const uint4 *>(vb + g));
                    }
                } else {
                    const float *kbase = static_cast<const float *>(kv.k) + hoff;
                    const float *vbase = static_cast<const float *>(kv.v) + hoff;
                    for (int i = tid; i < cached * (HD / 4); i += NCT) {
                        const int pp = i / (HD / 4), d4 = i - pp * (HD / 4);
                        reinterpret_cast<float4 *>(&sm->kv[0][pp][0])[d4] =
                            ldcg4(kbase + static_cast<size_t>(tp + pp) * HD + 4 * d4);
                        reinterpret_cast<float4 *>(&sm->kv[1][pp][0])[d4] =
                            ldcg4(vbase + static_cast<size_t>(tp + pp) * HD + 4 * d4);
                    }
                }
                named_sync();
            }
            if (active && ok) {
                for (int pp = sub; pp < nt; pp += npw) {
                    const int p = tp + pp;
                    if (p > L0 + cr) break;  // causal
                    float4 k, v;
                    if (p >= L0) {
                        k = *reinterpret_cast<const float4 *>(kn + (p - L0) * HD + 4 * lane);
                        v = *reinterpret_cast<const float4 *>(vn + (p - L0) * HD + 4 * lane);
                    } else if (KV16) {
                        k = h4_to_f4(ktile16 + pp * HD + 4 * lane);
                        v = h4_to_f4(vtile16 + pp * HD + 4 * lane);
                    } else {
                        k = *reinterpret_cast<const float4 *>(&sm->kv[0][pp][0] + 4 * lane);
                        v = *reinterpret_cast<const float4 *>(&sm->kv[1][pp][0] + 4 * lane);
                    }
                    float d = q.x * k.x;
                    d = fmaf(q.y, k.y, d);
                    d = fmaf(q.z, k.z, d);
                    d = fmaf(q.w, k.w, d);
                    d = warp_sum(d) * scale;
                    const float mn = fmaxf(m, d);
                    const float corr = expf(m - mn);
                    const float e = expf(d - mn);
                    l = l * corr + e;
                    o[0] = fmaf(e, v.x, o[0] * corr);
                    o[1] = fmaf(e, v.y, o[1] * corr);
                    o[2] = fmaf(e, v.z, o[2] * corr);
                    o[3] = fmaf(e, v.w, o[3] * corr);
                    m = mn;
                }
            }
        }
        // 3. merge the warps of each (row, q head), partial to global
        if (active) {
            float *ws = wst + warp * PSTRIDE;
            *reinterpret_cast<float4 *>(ws + 4 * lane) = make_float4(o[0], o[1], o[2], o[3]);
            if (lane == 0) {
                ws[HD] = m;
                ws[HD + 1] = l;
            }
        }
        named_sync();
        if (warp < nc) {
            const int r = warp >> 1, qq = warp & 1;
            const float *w0 = wst + (warp * npw) * PSTRIDE;
            // lane j brings warp j's (max, sum); the weights e^(m_j - M) are
            // computed in parallel and broadcast to the dims loop
            float mj = -INFINITY, lj = 0.f;
            if (lane < npw) {
                mj = w0[lane * PSTRIDE + HD];
                lj = w0[lane * PSTRIDE + HD + 1];
            }
            float M = mj;
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
            const float ej = (mj == -INFINITY || M == -INFINITY) ? 0.f : expf(mj - M);
            const float L = warp_sum(lj * ej);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
            for (int j = 0; j < npw; ++j) {
                const float e = __shfl_sync(0xffffffffu, ej, j);
                const float4 v = *reinterpret_cast<const float4 *>(w0 + j * PSTRIDE + 4 * lane);
                acc.x = fmaf(v.x, e, acc.x);
                acc.y = fmaf(v.y, e, acc.y);
                acc.z = fmaf(v.z, e, acc.z);
                acc.w = fmaf(v.w, e, acc.w);
            }
            if (head_path) {
                const float inv = 1.0f / L;
                *reinterpret_cast<float4 *>(sm->act + r * KO + qq * HD + 4 * lane) =
                    make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
            } else {
                float *pp = job->s.part + ((static_cast<size_t>(h * S + s) * RMAX + r) * 2 + qq) * PSTRIDE;
                *reinterpret_cast<float4 *>(pp + 4 * lane) = acc;
                if (lane == 0) {
                    pp[HD] = M;
                    pp[HD + 1] = L;
                }
            }
        }
        if (head_path) named_sync();
    }

    // ---------------------------------------------------------------- stack

    // one forward of a stack over R rows at positions L0..L0+R-1; layer 0's
    // input row r is in0[r] (+ in1[r]) (+ in2[r]).  The QKV rows reach the
    // attention, and the residual stream after a down projection reaches the
    // next layer's staging, as tagged words (no barrier); the O partials and
    // the SwiGLU rows, which every CTA reads whole, after a grid barrier, as
    // does the last layer's residual (read by the head).
    __device__ __forceinline__ void stack(const DStack &st, const DCtx &kv, int R, int L0, const float *const *in0,
                          const float *const *in1, const float *const *in2) {
        const Scratch &S = job->s;
        const float *xr[RMAX];
        for (int r = 0; r < RMAX; ++r) xr[r] = S.x + r * H;
        const int nsplit = att_splits(L0 + R, gridDim.x);
        const bool hp = per_head_path(L0 + R);
        unsigned xtag = 0;  // the residual handoff of the previous layer's down projection
        // ok is uniform over the CTA at the top of each layer: a failure sets
        // the CTA's abort flag, which the GEMV reads after its CTA barrier
        for (int l = 0; l < st.layers && ok; ++l) {
            const DLayer Ly = st.layer[l];
            // P1
            if (l == 0)
                stage_norm(in0, in1, in2, R, Ly.in_norm, true);
            else
                stage_norm(nullptr, nullptr, nullptr, R, Ly.in_norm, false, nullptr, S.x8, xtag);
            mark(10);
            const unsigned qtag = next_tag();
            cur_tag = qtag;
            gemv<H>(M_QKV, 0, R, E_TAGGED, reinterpret_cast<float *>(S.qkv), QKV_ROWS, st.eps);
            if (!ok) return;
            mark(11);
            prefetch_kv(kv, l, R, L0, hp);
            named_sync();  // thread 0's sm->kv_rows (the prefetched tile) for every thread
            // P2: the rows of this CTA's kv head, polled as they land
            attention(Ly, kv, l, R, L0, st.eps, hp, qtag);
            mark(21);
            if (hp) {
                // the O projection restricted to this head's columns, by head
                gemv<KO>(M_OH, 0, R, E_STORE, S.part, HKV * H, -1.f);
                mark(31);
                grid_sync(3);
                if (!ok) return;
                // P4: residual + the HKV partials (layer 0's residual is still
                // its input rows: they reach S.x with the down projection)
                if (l == 0)
                    stage_norm(in0, in1, in2, R, Ly.post_norm, true, S.part);
                else
                    stage_norm(xr, nullptr, nullptr, R, Ly.post_norm, true, S.part);
            } else {
                grid_sync(2);
                if (!ok) return;
                // P3
                stage_attn(R, nsplit);
                mark(30);
                gemv<QDIM>(M_O, 0, R, E_RESID, S.x, H, -1.f);
                mark(31);
                grid_sync(3);
                if (!ok) return;
                // P4
                stage_norm(xr, nullptr, nullptr, R, Ly.post_norm, false);
            }
            mark(40);
            gemv<H>(M_GU, 0, R, E_SWIGLU, S.act, INTER, st.eps);
            mark(41);
            grid_sync(4);
            if (!ok) return;
            // P5
            stage_copy(S.act, R, INTER);
            mark(50);
            const bool last = l + 1 == st.layers;
            if (!last) {
                xtag = next_tag();
                cur_tag = xtag;
                x8out = S.x8;
            }
            gemv<INTER>(M_D, 0, R, E_RESID, S.x, H, -1.f);
            x8out = nullptr;
            mark(51);
            if (last) grid_sync(5);
        }
    }

    // final norm of the last row, head GEMV; the normed state to hidden_out
    __device__ void head(const DStack &st, int R, int rows, int kind, float *hidden_out) {
        const Scratch &S = job->s;
        const float *last[1] = {S.x + (R - 1) * H};
        stage_norm(last, nullptr, nullptr, 1, st.final_norm, false);
        if (hidden_out && blockIdx.x == 0) {
            const float inv = norm_inv(0, st.eps);
            for (int i = tid; i < H; i += NCT) hidden_out[i] = sm->act[i] * inv;
        }
        mark(60);
        gemv<H>(M_HEAD, rows, 1, kind, S.logits, 0, st.eps);
        mark(61);
    }
};

// the program, walked by the producer
template <int WDT, class V>
__device__ void walk_stack(V &v, const DStack &st, int T) {
    const bool hp = per_head_path(T);
    for (int l = 0; l < st.layers; ++l) {
        const DLayer Ly = st.layer[l];
        v.matrix(Ly.wqkvh, M_QKV, 0, st.keep_l2);
        if (hp)
            v.matrix(Ly.woh, M_OH, 0, st.keep_l2);
        else
            v.matrix(Ly.wo, M_O, 0, st.keep_l2);
        v.matrix(Ly.wgu, M_GU, 0, st.keep_l2);
        v.matrix(Ly.wd, M_D, 0, st.keep_l2);
    }
}

template <int WDT>
__device__ void produce(Smem *sm, const Job &job) {
    Producer<WDT> p;
    p.sm = sm;
    if (job.mode == 0) {
        walk_stack<WDT>(p, job.st, job.L0 + job.rows);
        if (job.head_w) p.matrix(job.head_w, M_HEAD, job.head_rows, false);
    } else {
        // the contexts of the frame's calls (as the compute warps see them)
        const int tlen = job.fs->tlen;
        for (int g = 0; g < job.groups - 1; ++g) {
            walk_stack<WDT>(p, job.pst, g == 0 ? 2 : g + 2);
            p.matrix(job.pheads[g], M_HEAD, job.pvocab, false);
        }
        walk_stack<WDT>(p, job.tst, tlen + 1);
        p.matrix(job.theads, M_HEAD, job.tvocab, false);
    }
}

template <int WDT, int KV16>
__device__ void compute(Smem *sm, const Job &job) {
    Compute<WDT, KV16> c;
    c.sm = sm;
    c.job = &job;
    c.tid = threadIdx.x;
    c.warp = threadIdx.x >> 5;
    c.lane = threadIdx.x & 31;
    mat_slice(M_D, H, blockIdx.x, gridDim.x, c.c0, c.c1);  // the rows of its down-projection slice
    if (c.tid < M_FIXED) {
        const Mat m = static_cast<Mat>(c.tid);
        mat_slice(m, mat_rows(m, 0), blockIdx.x, gridDim.x, sm->slice[c.tid][0], sm->slice[c.tid][1]);
    }
    c.cta_sync();
    const Scratch &S = job.s;
    c.mark(1);
    if (job.mode == 0) {
        const float *in[RMAX];
        for (int r = 0; r < RMAX; ++r) in[r] = job.xin + r * H;
        c.stack(job.st, job.ctx, job.rows, job.L0, in, nullptr, nullptr);
        if (job.head_w && c.ok) {
            c.head(job.st, job.rows, job.head_rows, Compute<WDT, KV16>::E_HEAD, S.hidden);
        } else if (c.ok) {
            // no head: still return the normed last state
            const float *last[1] = {S.x + (job.rows - 1) * H};
            c.stage_norm(last, nullptr, nullptr, 1, job.st.final_norm, false);
            if (blockIdx.x == 0) {
                const float inv = c.norm_inv(0, job.st.eps);
                for (int i = c.tid; i < H; i += NCT) S.hidden[i] = sm->act[i] * inv;
            }
        }
    } else {
        FrameState *fs = job.fs;
        const int code0 = fs->next_code0;
        const int tlen = fs->tlen;
        const int step = fs->step;
        c.hist_now = fs->hist_len + 1;
        // the talker input starts as the code-0 embedding (talker.pas:669)
        const float *e0 = job.codec_emb + static_cast<size_t>(code0) * H;
        for (int i = c.c0 + c.tid; i < c.c1; i += NCT) S.xt[i] = e0[i];
        if (blockIdx.x == 0 && c.tid == 0) {
            job.seen[code0] = 1;
            fs->codes[0] = code0;
            if (job.codes_hist && step < job.codes_cap) job.codes_hist[step * job.groups] = code0;
        }
        // predictor: [talker state, codec_emb[code0]] then one row per group
        int code = code0;
        for (int g = 0; g < job.groups - 1 && c.ok; ++g) {
            const float *in[RMAX] = {nullptr, nullptr, nullptr, nullptr};
            int R;
            if (g == 0) {
                in[0] = S.hidden;
                in[1] = e0;
                R = 2;
            } else {
                in[0] = job.pred_emb + (static_cast<size_t>(g - 1) * job.pvocab + code) * H;
                R = 1;
            }
            const int L0 = g == 0 ? 0 : g + 1;
            c.stack(job.pst, job.pctx, R, L0, in, nullptr, nullptr);
            if (!c.ok) break;
            // greedy: the CTAs' argmax keys meet as tagged words (no barrier);
            // the row of pred_emb[g] the winner selects is prefetched into L2
            const bool tagged_keys = !job.samp.on && job.pvocab <= 4096;
            c.key_tag = tagged_keys ? c.next_tag() : 0u;
            c.next_rows = job.pred_emb + static_cast<size_t>(g) * job.pvocab * H;
            c.head(job.pst, R, job.pvocab, Compute<WDT, KV16>::E_HEAD, nullptr);
            const unsigned ktag = c.key_tag;
            c.key_tag = 0u;
            c.next_rows = nullptr;
            if (!c.ok) break;
            // ChooseCode (talker.pas:632-638): the draw (frame, group g + 1) or the argmax
            if (tagged_keys) {
                code = c.reduce_argmax_tagged(ktag);
            } else {
                c.grid_sync(6);
                if (!c.ok) break;
                code = job.samp.on ? c.sample_code(job.pvocab, job.samp, sample_uniform(job.seed, step, g + 1), false)
                                   : c.reduce_argmax();
            }
            if (!c.ok) break;
            if (blockIdx.x == 0 && c.tid == 0) {
                fs->codes[g + 1] = code;
                if (job.codes_hist && step < job.codes_cap) job.codes_hist[step * job.groups + g + 1] = code;
            }
            if (g + 1 < job.groups - 1) {
                // codes 1..14 enter the talker input now; code 15 at its staging
                const float *e = job.pred_emb + (static_cast<size_t>(g) * job.pvocab + code) * H;
                for (int i = c.c0 + c.tid; i < c.c1; i += NCT) S.xt[i] = S.xt[i] + e[i];
            }
        }
        if (c.ok) {
            const int G = job.groups;
            const float *in0[RMAX] = {S.xt, nullptr, nullptr, nullptr};
            const float *in1[RMAX] = {job.pred_emb + (static_cast<size_t>(G - 2) * job.pvocab + code) * H, nullptr,
                                      nullptr, nullptr};
            const float *tr = step < job.trailing_rows ? job.trailing + static_cast<size_t>(step) * H : job.tts_pad;
            const float *in2[RMAX] = {tr, nullptr, nullptr, nullptr};
            c.stack(job.tst, job.tctx, 1, tlen, in0, in1, in2);
            c.next_rows = job.codec_emb;  // the next frame starts from codec_emb[code 0]
            if (c.ok) c.head(job.tst, 1, job.tvocab, Compute<WDT, KV16>::E_HEAD0, S.hidden);
            c.next_rows = nullptr;
            if (c.ok) c.grid_sync(8);
            if (c.ok && blockIdx.x == 0 && (job.samp0.on || c.warp == 0)) {
                // ChooseCode0 of the next frame (its draw is (step + 1, 0));
                // the history holds this frame's code 0
                const int next = job.samp0.on ? c.sample_code(job.tvocab, job.samp0,
                                                              sample_uniform(job.seed, step + 1, 0), true)
                                              : c.reduce_argmax();
                if (c.tid == 0) {
                    fs->next_code0 = next;
                    fs->done = next == job.eos ? 1 : 0;
                    fs->step = step + 1;
                    fs->tlen = tlen + 1;
                    fs->hist_len = c.hist_now;
                }
            }
        }
    }
    if (job.trace && blockIdx.x == 0 && c.tid == 0) {
        c.mark(999);
        *job.trace_n = c.ntrace;
    }
    // a K/V prefetch still in flight (abort path) must land before exit
    c.cta_sync();
    if (c.tid == 0 && sm->kv_rows > 0) mbar_wait(&sm->kvbar, c.kv_phase, nullptr);
    // exit: the last CTA out resets the barrier counters for the next launch
    if (c.tid == 0 && c.ok) {
        __threadfence();
        if (atomicAdd(S.bar + 1, 1u) == gridDim.x - 1) {
            S.bar[0] = 0u;
            S.bar[1] = 0u;
            __threadfence();
        }
    }
}

template <int WDT, int KV16>
__global__ void __launch_bounds__(NTHREADS, 1) decode_kernel(const __grid_constant__ Job job) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem *sm = reinterpret_cast<Smem *>(smem_raw);
    if (threadIdx.x == 0) {
        for (int i = 0; i < NSTAGES; ++i) {
            mbar_init(&sm->full[i], 1);
            mbar_init(&sm->empty[i], NCW);
        }
        mbar_init(&sm->kvbar, 1);
        sm->abort_flag = 0;
        sm->issued = 0;
        sm->kv_rows = 0;
        sm->barflag[0] = sm->barflag[1] = sm->barflag[2] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (job.mode == 1 && job.fs->done) return;  // eos already chosen: nothing to do
    if (threadIdx.x / 32 == PRODUCER_WARP) {
        if (threadIdx.x % 32 == 0) produce<WDT>(sm, job);
    } else {
        compute<WDT, KV16>(sm, job);
    }
    // no bulk copy may be in flight when the CTA exits: after everyone is
    // done, wait for the last chunk issued into each slot (earlier chunks of
    // a slot completed before it was reused; normally all have landed)
    __syncthreads();
    if (threadIdx.x == 0) {
        const int issued = sm->issued;
        for (int s = 0; s < NSTAGES && s < issued; ++s) {
            const int last = s + NSTAGES * ((issued - 1 - s) / NSTAGES);
            mbar_wait(&sm->full[s], (last / NSTAGES) & 1, nullptr);
        }
    }
}

}  // namespace qtts
