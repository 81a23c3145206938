// qtts_decode.cuh -- the persistent decode kernel of libqtts (sm_100a).
//
// One cooperative launch runs either one TQwenLm.Forward of <= RMAX rows
// (mormot.ai.tts.qwen.lm.pas:391-408) or one whole TQwenTalker.NextFrame
// (mormot.ai.tts.qwen.talker.pas:640-681): 15 code-predictor steps with their
// heads and greedy argmax, the sum of the 16 code embeddings, the talker step,
// its head and ChooseCode0 for the next frame.
//
// Shape of the kernel
//  - one CTA per SM (grid = SM count, ~200 KB shared memory each), 16 warps:
//    warps 0..14 compute, warp 15 is the weight producer.
//  - the producer walks the same program as the compute warps and streams
//    this CTA's slice of every weight matrix, in program order, through a
//    ring of NSTAGES shared-memory stages with cp.async.bulk (global ->
//    shared, mbarrier complete_tx).  Weights never depend on activations, so
//    the stream runs ahead across grid barriers: the next matrix is already
//    in shared memory when its activations become ready.
//  - the compute warps run the phases of each layer, separated by grid
//    barriers (monotonic counter, release/acquire, bounded spin):
//      P1 rmsnorm + QKV GEMV -> qkv      | P2 q/k-norm + RoPE + KV append +
//      split-K attention, last split combines -> attn | P3 O GEMV + residual
//      | P4 rmsnorm + gate/up GEMV + SiLU*up -> act | P5 down GEMV + residual
//    then the final rmsnorm + head GEMV + argmax.
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
constexpr int NSTAGES = 6;
constexpr int ACT_FLOATS = RMAX * INTER;  // staged activations [R][K]
constexpr int MAX_ITEMS = 64;             // (row, 512-unit) items per stage
constexpr int PSTRIDE = 132;              // attention partial: o[128], m, l

constexpr int WDT_F32 = 0;
constexpr int WDT_Q8 = 1;

constexpr int ERR_TIMEOUT = 5;
constexpr int ERR_CAPACITY = 4;

constexpr unsigned long long WAIT_NS = 2000000000ull;  // 2 s per wait

__host__ __device__ constexpr int row_bytes(int wdt, int k) { return wdt == WDT_F32 ? k * 4 : k + k / 16; }

// ------------------------------------------------------------------ descriptors

struct DLayer {
    const uint8_t *wqkv, *wo, *wgu, *wd;
    const float *in_norm, *post_norm, *q_norm, *k_norm;
};

struct DStack {
    const DLayer *layer;  // device array
    int layers;
    float eps;
    const float *final_norm;
    int keep_l2;  // stream with L2 evict_last (weights that fit in L2)
};

struct DCtx {      // KV cache [layers][HKV][max_pos][HD], float32
    float *k, *v;
    int max_pos;
};

// scratch of one runner (one lm or one talker), all in global memory
struct Scratch {
    float *x;       // [RMAX][H] residual stream
    float *qkv;     // [RMAX][QKV_ROWS]
    float *attn;    // [RMAX][QDIM]
    float *act;     // [RMAX][INTER]
    float *part;    // [HKV*maxS][RMAX][2][PSTRIDE] attention partials
    unsigned *comb; // [HKV] split counters (last split combines)
    unsigned long long *arg;  // [grid] argmax keys
    unsigned *bar;  // [0] barrier counter, [1] exit counter
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
    FrameState *fs;
    int *codes_hist;         // [cap][groups] codes by frame index (may be NULL)
    int codes_cap;
    // both
    Scratch s;
    const float *rope_cos, *rope_sin;  // [rope_pos][HD/2]
    int rope_pos;
};

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
// bounded wait on an mbarrier phase; false on timeout
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, const volatile int *abort_flag) {
    if (mbar_test(b, parity)) return true;
    unsigned long long t0 = gtimer();
    while (!mbar_test(b, parity)) {
        if (abort_flag && *abort_flag) return false;
        if (gtimer() - t0 > WAIT_NS) return false;
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
__device__ __forceinline__ void named_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// int8 x4 (one 32-bit word) -> 4 exact floats: byte b^0x80 placed in the
// mantissa of 2^23, minus 2^23+128
__device__ __forceinline__ void dq4(uint32_t w, float &a, float &b, float &c, float &d) {
    uint32_t u = w ^ 0x80808080u;
    a = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650)) - 8388736.0f;
    b = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7651)) - 8388736.0f;
    c = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7652)) - 8388736.0f;
    d = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7653)) - 8388736.0f;
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

// ------------------------------------------------------------------ shared memory

struct __align__(128) Smem {
    uint8_t ring[NSTAGES][STAGE_BYTES];
    float act[ACT_FLOATS];
    float part[MAX_ITEMS * RMAX];
    float red[64];
    unsigned long long keys[NWARPS];
    uint64_t full[NSTAGES];
    uint64_t empty[NSTAGES];
    int abort_flag;
    int consumed;  // chunks released by the compute warps
    int bcast;
};

// ------------------------------------------------------------------ program walk

// Matrix phases in program order.  Both the producer and the compute warps
// call walk(); the producer issues the copies of each matrix slice, the
// compute warps do the work.  The order must not depend on data.
enum Mat { M_QKV, M_O, M_GU, M_D, M_HEAD };

__device__ __forceinline__ int mat_rows(Mat m, int head_rows) {
    switch (m) {
        case M_QKV: return QKV_ROWS;
        case M_O: return H;
        case M_GU: return GU_ROWS;
        case M_D: return H;
        default: return head_rows;
    }
}
__device__ __forceinline__ int mat_k(Mat m) {
    switch (m) {
        case M_O: return QDIM;
        case M_D: return INTER;
        default: return H;
    }
}
// rows [r0, r1) of an N-row matrix owned by CTA b of G (pairs for gate/up)
__device__ __forceinline__ void mat_slice(Mat m, int n, int b, int g, int &r0, int &r1) {
    if (m == M_GU) {
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
        }
    }
    // the copies issued but not consumed must land before the CTA exits
    __device__ void drain() {
        int c = *reinterpret_cast<volatile int *>(&sm->consumed);
        for (int n = c; n < seq; ++n) mbar_wait(&sm->full[n % NSTAGES], (n / NSTAGES) & 1, nullptr);
    }
};

// ------------------------------------------------------------------ compute

template <int WDT>
struct Compute {
    Smem *sm;
    const Job *job;
    int seq = 0;         // chunks consumed
    unsigned target = 0; // grid barrier target
    bool ok = true;
    int hist_now = 0;    // history length for ChooseCode0 (frame mode)
    int tid, warp, lane;

    __device__ void fail(int code, int where) {
        if (ok) {
            ok = false;
            atomicCAS(job->s.err, 0, code);
            atomicCAS(job->s.err + 1, 0, where);
            sm->abort_flag = 1;
        }
    }

    // grid-wide barrier among the compute warps of all CTAs
    __device__ void grid_sync(int where) {
        named_sync();
        if (tid == 0) {
            target += gridDim.x;
            if (ok) {
                __threadfence();
                atomicAdd(job->s.bar, 1u);
                volatile unsigned *c = job->s.bar;
                unsigned long long t0 = 0;
                int spins = 0;
                while (*c < target) {
                    if (*reinterpret_cast<volatile int *>(job->s.err) != 0) {
                        fail(ERR_TIMEOUT, where);
                        break;
                    }
                    if (++spins == 64) t0 = gtimer();
                    if (spins > 64 && gtimer() - t0 > WAIT_NS) {
                        fail(ERR_TIMEOUT, where);
                        break;
                    }
                }
                __threadfence();
            }
            sm->bcast = ok ? 0 : 1;
        }
        named_sync();
        if (sm->bcast) ok = false;
    }

    // ---------------------------------------------------------------- staging

    // act[r][0..H) = rmsnorm(row r) * w; rows given by up to 3 addends
    // (((a + b) + c), the summation order of TQwenTalker.NextFrame)
    __device__ void stage_norm(const float *const *a, const float *const *b, const float *const *c, int R,
                               const float *w, float eps, float *copy_to, int c0, int c1) {
        for (int r = 0; r < R; ++r) {
            float ss = 0.f;
            for (int i = tid; i < H; i += NCT) {
                float v = a[r][i];
                if (b && b[r]) v = v + b[r][i];
                if (c && c[r]) v = v + c[r][i];
                sm->act[r * H + i] = v;
                ss += v * v;
                if (copy_to && i >= c0 && i < c1) copy_to[r * H + i] = v;
            }
            ss = warp_sum(ss);
            if (lane == 0) sm->red[warp] = ss;
            named_sync();
            if (warp == 0) {
                float t = lane < NCW ? sm->red[lane] : 0.f;
                t = warp_sum(t);
                if (lane == 0) sm->red[32] = 1.0f / sqrtf(t / static_cast<float>(H) + eps);
            }
            named_sync();
            float inv = sm->red[32];
            for (int i = tid; i < H; i += NCT) sm->act[r * H + i] = w[i] * (sm->act[r * H + i] * inv);
            named_sync();
        }
    }
    __device__ void stage_copy(const float *src, int R, int k) {
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *d4 = reinterpret_cast<float4 *>(sm->act);
        for (int i = tid; i < R * k / 4; i += NCT) d4[i] = s4[i];
        named_sync();
    }

    // ---------------------------------------------------------------- GEMV

    // one (row, 512-unit) item: R dot products against the staged activations
    template <int K>
    __device__ __forceinline__ void item(const uint8_t *rowp, int u, int R, float *acc) {
#pragma unroll
        for (int r = 0; r < RMAX; ++r) acc[r] = 0.f;
        if (WDT == WDT_Q8) {
            const uint8_t *qp = rowp + u * 512;
            const __half *sp = reinterpret_cast<const __half *>(rowp + K) + u * 16;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                uint32_t w4 = *reinterpret_cast<const uint32_t *>(qp + 128 * g + 4 * lane);
                float d = __half2float(sp[4 * g + (lane >> 3)]);
                float q0, q1, q2, q3;
                dq4(w4, q0, q1, q2, q3);
#pragma unroll
                for (int r = 0; r < RMAX; ++r) {
                    if (r < R) {
                        float4 xv = *reinterpret_cast<const float4 *>(sm->act + r * K + u * 512 + 128 * g + 4 * lane);
                        float p = q0 * xv.x;
                        p = fmaf(q1, xv.y, p);
                        p = fmaf(q2, xv.z, p);
                        p = fmaf(q3, xv.w, p);
                        acc[r] = fmaf(d, p, acc[r]);
                    }
                }
            }
        } else {
            const float *wp = reinterpret_cast<const float *>(rowp) + u * 512;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                float4 w = *reinterpret_cast<const float4 *>(wp + 128 * g + 4 * lane);
#pragma unroll
                for (int r = 0; r < RMAX; ++r) {
                    if (r < R) {
                        float4 xv = *reinterpret_cast<const float4 *>(sm->act + r * K + u * 512 + 128 * g + 4 * lane);
                        float p = acc[r];
                        p = fmaf(w.x, xv.x, p);
                        p = fmaf(w.y, xv.y, p);
                        p = fmaf(w.z, xv.z, p);
                        p = fmaf(w.w, xv.w, p);
                        acc[r] = p;
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RMAX; ++r)
            if (r < R) acc[r] = warp_sum(acc[r]);
    }

    // Epilogue kinds
    enum Epi { E_STORE, E_ADD, E_SWIGLU, E_HEAD, E_HEAD0 };

    // GEMV over this CTA's slice of matrix m; activations already staged in
    // sm->act as [R][K].  Output per kind:
    //  E_STORE: out[r*ld + row] = y      E_ADD: out[r*ld + row] += y
    //  E_SWIGLU: out[r*ld + row/2] = silu(y_gate) * y_up
    //  E_HEAD / E_HEAD0: out[row] = y (R == 1), argmax key of the CTA in
    //  sm->keys[0]; E_HEAD0 applies ChooseCode0's processors to the key.
    template <int K>
    __device__ void gemv(Mat m, int head_rows, int R, int kind, float *out, int ld) {
        constexpr int UNITS = K / 512;
        const int rb = row_bytes(WDT, K);
        int n = mat_rows(m, head_rows);
        int r0, r1;
        mat_slice(m, n, blockIdx.x, gridDim.x, r0, r1);
        int sr = stage_rows(WDT, K, m);
        unsigned long long best = 0ull;
        for (int cr = r0; cr < r1; cr += sr) {
            int nr = min(sr, r1 - cr);
            int slot = seq % NSTAGES;
            uint32_t par = (seq / NSTAGES) & 1;
            // every thread waits (bounded); a timeout raises abort_flag, read
            // by all after the named barrier below, so the exit is uniform
            bool got = ok && mbar_wait(&sm->full[slot], par, &sm->abort_flag);
            if (!got) fail(ERR_TIMEOUT, 100 + m);
            const uint8_t *base = sm->ring[slot];
            int items = got ? nr * UNITS : 0;
            for (int it = warp; it < items; it += NCW) {
                int row = it / UNITS, u = it - row * UNITS;
                float acc[RMAX];
                item<K>(base + row * rb, u, R, acc);
                if (lane == 0) {
#pragma unroll
                    for (int r = 0; r < RMAX; ++r)
                        if (r < R) sm->part[it * RMAX + r] = acc[r];
                }
            }
            named_sync();
            if (*reinterpret_cast<volatile int *>(&sm->abort_flag)) {
                ok = false;
                return;
            }
            if (tid == 0) {
                mbar_arrive(&sm->empty[slot]);
                sm->consumed = seq + 1;
            }
            ++seq;
            if (kind == E_SWIGLU) {
                int npairs = nr / 2;
                for (int idx = tid; idx < npairs * R; idx += NCT) {
                    int p = idx / R, r = idx - p * R;
                    float g = 0.f, v = 0.f;
#pragma unroll
                    for (int u = 0; u < UNITS; ++u) {
                        g += sm->part[((2 * p) * UNITS + u) * RMAX + r];
                        v += sm->part[((2 * p + 1) * UNITS + u) * RMAX + r];
                    }
                    float s = g / (1.0f + expf(-g));
                    out[r * ld + (cr + 2 * p) / 2] = s * v;
                }
            } else {
                for (int idx = tid; idx < nr * R; idx += NCT) {
                    int row = idx / R, r = idx - row * R;
                    float y = 0.f;
#pragma unroll
                    for (int u = 0; u < UNITS; ++u) y += sm->part[(row * UNITS + u) * RMAX + r];
                    int orow = cr + row;
                    if (kind == E_STORE) {
                        out[r * ld + orow] = y;
                    } else if (kind == E_ADD) {
                        out[r * ld + orow] = out[r * ld + orow] + y;
                    } else {
                        out[orow] = y;
                        float w = y;
                        if (kind == E_HEAD0) w = choose0_value(orow, y);
                        unsigned long long k = argkey(w, orow);
                        best = k > best ? k : best;
                    }
                }
            }
            named_sync();
        }
        if (kind == E_HEAD || kind == E_HEAD0) {
            // CTA-wide max of the keys
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
                best = t > best ? t : best;
            }
            if (lane == 0) sm->keys[warp] = best;
            named_sync();
            if (tid == 0) {
                unsigned long long b = 0ull;
                for (int w = 0; w < NCW; ++w) b = sm->keys[w] > b ? sm->keys[w] : b;
                job->s.arg[blockIdx.x] = b;
            }
        }
    }

    // TQwenTalker.ChooseCode0 (talker.pas:595-630), greedy, for one logit:
    // the last 1024 ids forbidden but eos, eos forbidden before 2 frames,
    // repetition penalty once per distinct code already returned
    __device__ __forceinline__ float choose0_value(int i, float s) {
        int vocab = job->tvocab;
        if (i >= vocab - 1024 && i != job->eos) return -INFINITY;
        if (i == job->eos && hist_now < 2) return -INFINITY;
        if (job->penalty != 1.0f && job->seen[i]) return s > 0.f ? __fdiv_rn(s, job->penalty) : s * job->penalty;
        return s;
    }

    // after a grid barrier: the winning index over all CTAs' keys
    __device__ int reduce_argmax() {
        unsigned long long b = 0ull;
        for (int i = lane; i < static_cast<int>(gridDim.x); i += 32) {
            unsigned long long k = *reinterpret_cast<volatile unsigned long long *>(job->s.arg + i);
            b = k > b ? k : b;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
            b = t > b ? t : b;
        }
        return key_index(b);
    }

    // ---------------------------------------------------------------- attention

    // P2: per (kv head h, split s): q/k norm + RoPE, KV append (split 0),
    // online-softmax attention over positions [p0, p1), partials to global;
    // the last split of head h to finish combines them into attn.
    __device__ void attention(const DLayer &Ly, const DCtx &kv, int layer, int R, int L0, float eps) {
        const int T = L0 + R;
        int S = min(static_cast<int>(gridDim.x) / HKV, (T + 15) / 16);
        if (S < 1) S = 1;
        const int C = (T + S - 1) / S;
        const int item_id = blockIdx.x;
        if (item_id >= HKV * S) return;
        const int h = item_id / S, s = item_id - h * S;
        const int p0 = s * C, p1 = min(T, p0 + C);
        // shared layout inside sm->act: q[R][2][HD] | kn[R][HD] | vn[R][HD] | kt[32][HD] | vt[32][HD]
        float *qs = sm->act;
        float *kn = qs + RMAX * 2 * HD;
        float *vn = kn + RMAX * HD;
        float *kt = vn + RMAX * HD;
        float *vt = kt + 32 * HD;
        const int half = HD / 2;
        // 1. q (heads 2h, 2h+1), k, v of the new rows: norm + RoPE
        for (int vec = warp; vec < 4 * R; vec += NCW) {
            int r = vec >> 2, t = vec & 3;  // t: 0,1 = q heads, 2 = k, 3 = v
            const float *src = job->s.qkv + r * QKV_ROWS;
            int off = t < 2 ? (2 * h + t) * HD : (t == 2 ? QDIM + h * HD : QDIM + KVDIM + h * HD);
            float4 x = *reinterpret_cast<const float4 *>(src + off + 4 * lane);
            float y[4] = {x.x, x.y, x.z, x.w};
            if (t < 3) {
                const float *nw = t < 2 ? Ly.q_norm : Ly.k_norm;
                float ss = warp_sum(y[0] * y[0] + y[1] * y[1] + y[2] * y[2] + y[3] * y[3]);
                float inv = 1.0f / sqrtf(ss / static_cast<float>(HD) + eps);
#pragma unroll
                for (int j = 0; j < 4; ++j) y[j] = nw[4 * lane + j] * (y[j] * inv);
                const int pos = L0 + r;
                const float *cs = job->rope_cos + static_cast<size_t>(pos) * half;
                const float *sn = job->rope_sin + static_cast<size_t>(pos) * half;
                float o[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float partner = __shfl_xor_sync(0xffffffffu, y[j], 16);
                    int e = 4 * lane + j;
                    if (e < half)
                        o[j] = y[j] * cs[e] - partner * sn[e];
                    else
                        o[j] = y[j] * cs[e - half] + partner * sn[e - half];
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) y[j] = o[j];
            }
            float *dst = t < 2 ? qs + (r * 2 + t) * HD : (t == 2 ? kn + r * HD : vn + r * HD);
            *reinterpret_cast<float4 *>(dst + 4 * lane) = make_float4(y[0], y[1], y[2], y[3]);
            if (s == 0 && t >= 2) {
                float *cache = (t == 2 ? kv.k : kv.v) +
                               ((static_cast<size_t>(layer) * HKV + h) * kv.max_pos + (L0 + r)) * HD;
                *reinterpret_cast<float4 *>(cache + 4 * lane) = make_float4(y[0], y[1], y[2], y[3]);
            }
        }
        named_sync();
        // 2. online softmax over [p0, p1), 32-position tiles
        const float scale = 1.0f / sqrtf(static_cast<float>(HD));
        float m = -INFINITY, l = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
        const int combo = warp;  // (r, qh) = (combo >> 1, combo & 1)
        const int cr = combo >> 1, cq = combo & 1;
        const float *kbase = kv.k + (static_cast<size_t>(layer) * HKV + h) * kv.max_pos * HD;
        const float *vbase = kv.v + (static_cast<size_t>(layer) * HKV + h) * kv.max_pos * HD;
        for (int tp = p0; tp < p1; tp += 32) {
            int nt = min(32, p1 - tp);
            for (int i = tid; i < nt * (HD / 4); i += NCT) {
                int pp = i / (HD / 4), d4 = i - pp * (HD / 4);
                int p = tp + pp;
                float4 kk, vv;
                if (p < L0) {
                    kk = reinterpret_cast<const float4 *>(kbase + static_cast<size_t>(p) * HD)[d4];
                    vv = reinterpret_cast<const float4 *>(vbase + static_cast<size_t>(p) * HD)[d4];
                } else {
                    kk = reinterpret_cast<const float4 *>(kn + (p - L0) * HD)[d4];
                    vv = reinterpret_cast<const float4 *>(vn + (p - L0) * HD)[d4];
                }
                reinterpret_cast<float4 *>(kt + pp * HD)[d4] = kk;
                reinterpret_cast<float4 *>(vt + pp * HD)[d4] = vv;
            }
            named_sync();
            if (combo < 2 * R) {
                float4 q = *reinterpret_cast<const float4 *>(qs + (cr * 2 + cq) * HD + 4 * lane);
                for (int pp = 0; pp < nt; ++pp) {
                    int p = tp + pp;
                    if (p > L0 + cr) break;  // causal
                    float4 k = *reinterpret_cast<const float4 *>(kt + pp * HD + 4 * lane);
                    float d = q.x * k.x;
                    d = fmaf(q.y, k.y, d);
                    d = fmaf(q.z, k.z, d);
                    d = fmaf(q.w, k.w, d);
                    d = warp_sum(d) * scale;
                    float mn = fmaxf(m, d);
                    float corr = expf(m - mn);
                    float e = expf(d - mn);
                    l = l * corr + e;
                    float4 v = *reinterpret_cast<const float4 *>(vt + pp * HD + 4 * lane);
                    o[0] = fmaf(e, v.x, o[0] * corr);
                    o[1] = fmaf(e, v.y, o[1] * corr);
                    o[2] = fmaf(e, v.z, o[2] * corr);
                    o[3] = fmaf(e, v.w, o[3] * corr);
                    m = mn;
                }
            }
            named_sync();
        }
        // 3. partials
        if (combo < 2 * R) {
            float *pp = job->s.part + ((static_cast<size_t>(item_id) * RMAX + cr) * 2 + cq) * PSTRIDE;
            *reinterpret_cast<float4 *>(pp + 4 * lane) = make_float4(o[0], o[1], o[2], o[3]);
            if (lane == 0) {
                pp[HD] = m;
                pp[HD + 1] = l;
            }
        }
        __threadfence();
        named_sync();
        if (tid == 0) sm->bcast = (atomicAdd(job->s.comb + h, 1u) == static_cast<unsigned>(S - 1));
        named_sync();
        if (!sm->bcast) return;
        // 4. last split of head h: combine
        __threadfence();
        for (int idx = tid; idx < R * 2 * HD; idx += NCT) {
            int r = idx / (2 * HD), rem = idx - r * 2 * HD, q = rem / HD, d = rem - q * HD;
            float M = -INFINITY;
            for (int j = 0; j < S; ++j) {
                const volatile float *pj =
                    job->s.part + ((static_cast<size_t>(h * S + j) * RMAX + r) * 2 + q) * PSTRIDE;
                M = fmaxf(M, pj[HD]);
            }
            float L = 0.f, acc = 0.f;
            for (int j = 0; j < S; ++j) {
                const volatile float *pj =
                    job->s.part + ((static_cast<size_t>(h * S + j) * RMAX + r) * 2 + q) * PSTRIDE;
                float w = expf(pj[HD] - M);
                L += pj[HD + 1] * w;
                acc += pj[d] * w;
            }
            job->s.attn[r * QDIM + (2 * h + q) * HD + d] = acc / L;
        }
        if (tid == 0) job->s.comb[h] = 0u;
    }

    // ---------------------------------------------------------------- stack

    // one forward of a stack over R rows at positions L0..L0+R-1; layer 0's
    // input row r is in0[r] (+ in1[r]) (+ in2[r])
    __device__ void stack(const DStack &st, const DCtx &kv, int R, int L0, const float *const *in0,
                          const float *const *in1, const float *const *in2) {
        const Scratch &S = job->s;
        int c0, c1;
        mat_slice(M_O, H, blockIdx.x, gridDim.x, c0, c1);
        const float *xr[RMAX];
        for (int r = 0; r < RMAX; ++r) xr[r] = S.x + r * H;
        for (int l = 0; l < st.layers && ok; ++l) {
            const DLayer Ly = st.layer[l];
            // P1
            if (l == 0)
                stage_norm(in0, in1, in2, R, Ly.in_norm, st.eps, S.x, c0, c1);
            else
                stage_norm(xr, nullptr, nullptr, R, Ly.in_norm, st.eps, nullptr, 0, 0);
            gemv<H>(M_QKV, 0, R, E_STORE, S.qkv, QKV_ROWS);
            grid_sync(1);
            if (!ok) return;
            // P2
            attention(Ly, kv, l, R, L0, st.eps);
            grid_sync(2);
            if (!ok) return;
            // P3
            stage_copy(S.attn, R, QDIM);
            gemv<QDIM>(M_O, 0, R, E_ADD, S.x, H);
            grid_sync(3);
            if (!ok) return;
            // P4
            stage_norm(xr, nullptr, nullptr, R, Ly.post_norm, st.eps, nullptr, 0, 0);
            gemv<H>(M_GU, 0, R, E_SWIGLU, S.act, INTER);
            grid_sync(4);
            if (!ok) return;
            // P5
            stage_copy(S.act, R, INTER);
            gemv<INTER>(M_D, 0, R, E_ADD, S.x, H);
            grid_sync(5);
        }
    }

    // final norm of the last row, head GEMV; the normed state to `hidden`
    __device__ void head(const DStack &st, int R, int rows, int kind, float *hidden_out) {
        const Scratch &S = job->s;
        const float *last[1] = {S.x + (R - 1) * H};
        stage_norm(last, nullptr, nullptr, 1, st.final_norm, st.eps, nullptr, 0, 0);
        if (hidden_out && blockIdx.x == 0)
            for (int i = tid; i < H; i += NCT) hidden_out[i] = sm->act[i];
        gemv<H>(M_HEAD, rows, 1, kind, S.logits, 0);
    }
};

// the program, walked by both roles
template <int WDT, class V>
__device__ void walk_stack(V &v, const DStack &st) {
    for (int l = 0; l < st.layers; ++l) {
        const DLayer Ly = st.layer[l];
        v.matrix(Ly.wqkv, M_QKV, 0, st.keep_l2);
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
        walk_stack<WDT>(p, job.st);
        if (job.head_w) p.matrix(job.head_w, M_HEAD, job.head_rows, false);
    } else {
        for (int g = 0; g < job.groups - 1; ++g) {
            walk_stack<WDT>(p, job.pst);
            p.matrix(job.pheads[g], M_HEAD, job.pvocab, false);
        }
        walk_stack<WDT>(p, job.tst);
        p.matrix(job.theads, M_HEAD, job.tvocab, false);
    }
    p.drain();
}

template <int WDT>
__device__ void compute(Smem *sm, const Job &job) {
    Compute<WDT> c;
    c.sm = sm;
    c.job = &job;
    c.tid = threadIdx.x;
    c.warp = threadIdx.x >> 5;
    c.lane = threadIdx.x & 31;
    const Scratch &S = job.s;
    if (job.mode == 0) {
        const float *in[RMAX];
        for (int r = 0; r < RMAX; ++r) in[r] = job.xin + r * H;
        c.stack(job.st, job.ctx, job.rows, job.L0, in, nullptr, nullptr);
        if (job.head_w && c.ok) c.head(job.st, job.rows, job.head_rows, Compute<WDT>::E_HEAD, S.hidden);
        else if (c.ok) {
            // no head: still return the normed last state
            const float *last[1] = {S.x + (job.rows - 1) * H};
            c.stage_norm(last, nullptr, nullptr, 1, job.st.final_norm, job.st.eps, nullptr, 0, 0);
            if (blockIdx.x == 0)
                for (int i = c.tid; i < H; i += NCT) S.hidden[i] = sm->act[i];
        }
    } else {
        FrameState *fs = job.fs;
        const int code0 = fs->next_code0;
        const int tlen = fs->tlen;
        c.hist_now = fs->hist_len + 1;
        int c0, c1;
        mat_slice(M_O, H, blockIdx.x, gridDim.x, c0, c1);
        // the talker input starts as the code-0 embedding (talker.pas:669)
        const float *e0 = job.codec_emb + static_cast<size_t>(code0) * H;
        for (int i = c0 + c.tid; i < c1; i += NCT) S.xt[i] = e0[i];
        if (blockIdx.x == 0 && c.tid == 0) {
            job.seen[code0] = 1;
            fs->codes[0] = code0;
            if (job.codes_hist && fs->step < job.codes_cap) job.codes_hist[fs->step * job.groups] = code0;
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
            int L0 = g == 0 ? 0 : g + 1;
            c.stack(job.pst, job.pctx, R, L0, in, nullptr, nullptr);
            if (!c.ok) break;
            c.head(job.pst, R, job.pvocab, Compute<WDT>::E_HEAD, nullptr);
            c.grid_sync(6);
            if (!c.ok) break;
            code = c.reduce_argmax();
            if (blockIdx.x == 0 && c.tid == 0) {
                fs->codes[g + 1] = code;
                if (job.codes_hist && fs->step < job.codes_cap) job.codes_hist[fs->step * job.groups + g + 1] = code;
            }
            if (g + 1 < job.groups - 1) {
                // codes 1..14 enter the talker input now; code 15 at its staging
                const float *e = job.pred_emb + (static_cast<size_t>(g) * job.pvocab + code) * H;
                for (int i = c0 + c.tid; i < c1; i += NCT) S.xt[i] = S.xt[i] + e[i];
            }
        }
        if (c.ok) {
            const int G = job.groups;
            const float *in0[RMAX] = {S.xt, nullptr, nullptr, nullptr};
            const float *in1[RMAX] = {job.pred_emb + (static_cast<size_t>(G - 2) * job.pvocab + code) * H, nullptr,
                                      nullptr, nullptr};
            const int step = fs->step;
            const float *tr = step < job.trailing_rows ? job.trailing + static_cast<size_t>(step) * H : job.tts_pad;
            const float *in2[RMAX] = {tr, nullptr, nullptr, nullptr};
            c.stack(job.tst, job.tctx, 1, tlen, in0, in1, in2);
            if (c.ok) c.head(job.tst, 1, job.tvocab, Compute<WDT>::E_HEAD0, S.hidden);
            if (c.ok) c.grid_sync(8);
            if (c.ok && blockIdx.x == 0 && c.warp == 0) {
                // ChooseCode0 of the next frame; the history holds this frame's code 0
                int next = c.reduce_argmax();
                if (c.lane == 0) {
                    fs->next_code0 = next;
                    fs->done = next == job.eos ? 1 : 0;
                    fs->step = step + 1;
                    fs->tlen = tlen + 1;
                    fs->hist_len = c.hist_now;
                }
            }
        }
    }
    // exit: the last CTA out resets the barrier counters for the next launch
    named_sync();
    if (c.tid == 0 && c.ok) {
        __threadfence();
        if (atomicAdd(S.bar + 1, 1u) == gridDim.x - 1) {
            S.bar[0] = 0u;
            S.bar[1] = 0u;
            __threadfence();
        }
    }
}

template <int WDT>
__global__ void __launch_bounds__(NTHREADS, 1) decode_kernel(const Job job) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem *sm = reinterpret_cast<Smem *>(smem_raw);
    if (threadIdx.x == 0) {
        for (int i = 0; i < NSTAGES; ++i) {
            mbar_init(&sm->full[i], 1);
            mbar_init(&sm->empty[i], 1);
        }
        sm->abort_flag = 0;
        sm->consumed = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (job.mode == 1 && job.fs->done) return;  // eos already chosen: nothing to do
    if (threadIdx.x / 32 == PRODUCER_WARP) {
        if (threadIdx.x % 32 == 0) produce<WDT>(sm, job);
    } else {
        compute<WDT>(sm, job);
    }
}

}  // namespace qtts
