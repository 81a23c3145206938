// qtts_sample.cuh -- the draw of one code from its logits (sm_100a): the
// sampling mode of TQwenTalker's choices (talker.pas:626-629 for code 0,
// 632-638 for the predictor's codes), whose TInferSampler lives in the
// mormot2-ai submodule.  Its steps follow the logits warpers of transformers'
// generate, which the reference's options mirror (generation_config:
// temperature, top_k, top_p; talker.pas:203-229):
//   z = logit / temperature;
//   keep the values >= the top_k-th largest z (ties kept, -inf never);
//   order them by (z desc, index asc);
//   keep the nucleus: a value stays while the probability mass before it
//   is < top_p (the first always stays);
//   draw by inverse CDF: the first value whose running sum of
//   exp(z - z_max), in that order, exceeds u * (the nucleus' sum).
// u is counter-based: splitmix64 (Vigna's published finaliser) of
// seed + (16 * step + group + 1) * 0x9E3779B97F4A7C15, top 24 bits / 2^24,
// so a draw depends only on (seed, frame, code group).  The running sums are
// taken by one thread in candidate order, so that a CPU restatement repeats
// them exactly.
//
// One CTA (NT threads, named barrier 1) draws: a radix select (4 passes of
// 8 bits over the orderable keys, two histograms used in turn so that one
// is cleared while the other is scanned) finds the top_k-th largest value,
// the candidates are gathered one atomic per warp (ballot) and ranked by
// counting, the weights exp(z - z_max) are computed in parallel and summed
// by thread 0.
#pragma once
#include <stdint.h>

namespace qtts {

constexpr int SAMPLE_MAX_K = 64;      // top_k limit (generation_config: 50)
constexpr int SAMPLE_MAX_CAND = 128;  // candidates kept (the top_k and ties at the threshold)
constexpr int SAMPLE_MAX_V = 4096;    // logits of one draw

struct SampleParams {
    int on;             // 0: greedy (the first maximum)
    float temperature;  // > 0
    int top_k;          // 1 .. SAMPLE_MAX_K
    float top_p;        // (0, 1]
};

__host__ __device__ inline uint64_t sample_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// the uniform of draw (step, group) of the stream `seed`, in [0, 1)
__host__ __device__ inline float sample_uniform(uint64_t seed, int step, int group) {
    const uint64_t c = static_cast<uint64_t>(step) * 16u + static_cast<uint64_t>(group) + 1u;
    const uint64_t z = sample_mix64(seed + c * 0x9E3779B97F4A7C15ull);
    return static_cast<float>(z >> 40) * (1.0f / 16777216.0f);
}

struct SampleScratch {
    unsigned hist[2][256];  // the radix passes alternate between the two
    unsigned cnt, sel, rem;
    int code;
    alignas(8) unsigned ckey[SAMPLE_MAX_CAND];
    int cidx[SAMPLE_MAX_CAND];
    int sidx[SAMPLE_MAX_CAND];
    float sz[SAMPLE_MAX_CAND];
    float sw[SAMPLE_MAX_CAND];
    unsigned long long pk[SAMPLE_MAX_CAND];  // (key, ~index) of the candidates, for the ranking
};

// orderable key of a float (larger value, larger key) and back
__device__ __forceinline__ unsigned sample_key(float z) {
    const unsigned b = __float_as_uint(z);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float sample_unkey(unsigned k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

template <int NT>
__device__ __forceinline__ void sample_sync() {
    __syncwarp();
    asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
}

// The code drawn from values load(0 .. V-1) (logits after the processors)
// with the uniform u; every one of the NT threads calls it and gets the
// code.  V <= SAMPLE_MAX_V; ss in shared memory.
template <int NT, class Load>
__device__ int sample_draw(Load load, int V, const SampleParams &p, float u, SampleScratch *ss, int tid) {
    constexpr int KPT = (SAMPLE_MAX_V + NT - 1) / NT;
    const int lane = tid & 31;
    const unsigned key_ninf = sample_key(-INFINITY);
    unsigned key[KPT];
#pragma unroll
    for (int j = 0; j < KPT; ++j) {
        const int i = tid + j * NT;
        key[j] = i < V ? sample_key(load(i) / p.temperature) : 0u;
    }
    // radix select of the top_k-th largest key, 8 bits a pass from the top
    unsigned prefix = 0u, mask = 0u;
    unsigned rem = static_cast<unsigned>(min(max(p.top_k, 1), V));
    for (int b = tid; b < 512; b += NT) (&ss->hist[0][0])[b] = 0u;
    sample_sync<NT>();
    for (int d = 3; d >= 0; --d) {
        unsigned *hist = ss->hist[d & 1];
#pragma unroll
        for (int j = 0; j < KPT; ++j)
            if (tid + j * NT < V && (key[j] & mask) == prefix) atomicAdd(&hist[(key[j] >> (8 * d)) & 255u], 1u);
        sample_sync<NT>();
        // the other histogram is cleared for the next pass while warp 0 scans this one
        for (int b = tid - 32; b >= 0 && b < 256; b += NT - 32) ss->hist[(d & 1) ^ 1][b] = 0u;
        if (tid < 32) {
            // lane: bins 255 - 8 lane - q, q = 0..7 (descending); counts of
            // the bins above as an exclusive prefix over the lanes
            unsigned c[8], tot = 0u;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                c[q] = hist[255 - 8 * lane - q];
                tot += c[q];
            }
            unsigned incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            const unsigned excl = incl - tot;
            if (excl < rem && rem <= incl) {
                unsigned acc = excl;
                for (int q = 0; q < 8; ++q) {
                    if (acc + c[q] >= rem) {
                        ss->sel = static_cast<unsigned>(255 - 8 * lane - q);
                        ss->rem = rem - acc;
                        break;
                    }
                    acc += c[q];
                }
            }
        }
        sample_sync<NT>();
        prefix |= ss->sel << (8 * d);
        mask |= 0xFFu << (8 * d);
        rem = ss->rem;
    }
    // candidates: keys >= the threshold, -inf excluded; one atomic per
    // warp and pass (ballot), each lane at its prefix in the warp's run
    if (tid == 0) ss->cnt = 0u;
    sample_sync<NT>();
#pragma unroll
    for (int j = 0; j < KPT; ++j) {
        const int i = tid + j * NT;
        const bool c = i < V && key[j] >= prefix && key[j] != key_ninf;
        const unsigned b = __ballot_sync(0xffffffffu, c);
        if (b) {
            unsigned base = 0u;
            if (lane == __ffs(b) - 1) base = atomicAdd(&ss->cnt, static_cast<unsigned>(__popc(b)));
            base = __shfl_sync(0xffffffffu, base, __ffs(b) - 1);
            const unsigned s = base + static_cast<unsigned>(__popc(b & ((1u << lane) - 1u)));
            if (c && s < SAMPLE_MAX_CAND) {
                ss->ckey[s] = key[j];
                ss->cidx[s] = i;
            }
        }
    }
    sample_sync<NT>();
    const int n = static_cast<int>(ss->cnt);
    if (n == 0) return 0;  // every value -inf: the first maximum
    if (n > SAMPLE_MAX_CAND) {
        // more ties at the threshold than the candidates kept (not a case of
        // real logits): the first maximum of z, the same in every CTA
        unsigned long long best = 0ull;
#pragma unroll
        for (int j = 0; j < KPT; ++j) {
            const int i = tid + j * NT;
            if (i < V) {
                const unsigned long long k = (static_cast<unsigned long long>(key[j]) << 32) | (0xFFFFFFFFu - i);
                best = k > best ? k : best;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
            best = t > best ? t : best;
        }
        if (tid == 0) *reinterpret_cast<unsigned long long *>(ss->ckey) = 0ull;
        sample_sync<NT>();
        if (lane == 0) atomicMax(reinterpret_cast<unsigned long long *>(ss->ckey), best);
        sample_sync<NT>();
        const unsigned long long b = *reinterpret_cast<const volatile unsigned long long *>(ss->ckey);
        sample_sync<NT>();
        return static_cast<int>(0xFFFFFFFFu - static_cast<unsigned>(b & 0xFFFFFFFFull));
    }
    // rank under (z desc, index asc): (key, ~index) as one 64-bit value,
    // larger first; the loops stay rolled (the draw runs between layers,
    // where its code is fetched cold: a smaller body is the faster one)
    unsigned long long *pk = ss->pk;
    for (int c = tid; c < n; c += NT)
        pk[c] = (static_cast<unsigned long long>(ss->ckey[c]) << 32) | (0xFFFFFFFFu - static_cast<unsigned>(ss->cidx[c]));
    sample_sync<NT>();
    for (int c = tid; c < n; c += NT) {
        const unsigned long long kc = pk[c];
        int r = 0;
        for (int m = 0; m < n; ++m) r += pk[m] > kc ? 1 : 0;
        ss->sidx[r] = static_cast<int>(0xFFFFFFFFu - static_cast<unsigned>(kc));
        ss->sz[r] = sample_unkey(static_cast<unsigned>(kc >> 32));
    }
    sample_sync<NT>();
    const float mx = ss->sz[0];
    for (int c = tid; c < n; c += NT) ss->sw[c] = expf(ss->sz[c] - mx);
    sample_sync<NT>();
    if (tid == 0) {
        float total = 0.0f;
        for (int c = 0; c < n; ++c) total += ss->sw[c];
        int nk = n;
        if (p.top_p < 1.0f) {
            float acc = 0.0f;
            for (int c = 0; c < n; ++c) {
                if (c > 0 && acc / total >= p.top_p) {
                    nk = c;
                    break;
                }
                acc += ss->sw[c];
            }
        }
        float wsum = total;
        if (nk < n) {
            wsum = 0.0f;
            for (int c = 0; c < nk; ++c) wsum += ss->sw[c];
        }
        const float target = u * wsum;
        float acc = 0.0f;
        int code = ss->sidx[nk - 1];
        for (int c = 0; c < nk; ++c) {
            acc += ss->sw[c];
            if (acc > target) {
                code = ss->sidx[c];
                break;
            }
        }
        ss->code = code;
    }
    sample_sync<NT>();
    return ss->code;
}

}  // namespace qtts
