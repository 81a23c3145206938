// qtts_codec.cuh -- the 12 Hz decoder of Qwen3-TTS on the device (sm_100a):
// TQwenCodec (src/tts/mormot.ai.tts.qwen.codec.pas), 16 codes per frame ->
// 1920 samples at 24 kHz, frame by frame, every layer keeping its causal
// history on the device (convolution rows, the attention's keys and values)
// so that frames decoded in successive calls give the samples of one call.
//
// Layout: activations float32, rows = time steps, columns = channels (as the
// reference).  Every convolution is a product of its im2col rows with the
// weights [out][in * K] (transposed convolutions with weights re-laid
// [stride * out][taps * in] at load, as TQwenTransConv.Create,
// codec.pas:366-396), and so are the linear layers: all on one tcgen05
// product kernel with float32 accuracy (3xTF32); the rest are row and
// element kernels.  Included at the end of qtts_api.cu (it uses the file's
// safetensors helpers and error reporting).
#pragma once

namespace qcodec {

constexpr int CG = 16, CB = 2048, CODE_DIM = 256, QUANT_DIM = 512, LATENT = 1024;
constexpr int TF_DIM = 512, TF_HEADS = 16, TF_HD = 64, TF_QKV = TF_HEADS * TF_HD, TF_MLP = 1024, TF_LAYERS = 8;
constexpr int TF_WINDOW = 72, DEC_DIM = 1536, FRAME_SAMPLES = 1920;

// The K chunk of a split GEMM: a K longer than this is cut into chunks of
// KC, each chunk's products summed by its own CTAs into a partial, and the
// partials added in chunk order by splitk_reduce_kernel.  The cut depends on
// K alone, never on the rows of a call, so frames decoded one call at a time
// still give exactly the samples of one call.
constexpr int KC = 256;

// y[M][N] = a[M][K] . w[N][K]^T (+ bias) on the 5th-generation tensor cores
// with float32 accuracy ("3xTF32"): every operand is split into its tf32
// part (10-bit mantissa, rounded to nearest) and the float32 rest, x = hi +
// lo, and the product is hi_a hi_w + hi_a lo_w + lo_a hi_w (tcgen05.mma
// kind::tf32, f32 accumulation in TMEM); the dropped lo_a lo_w is below
// 2^-20 of |a w|, and each lo enters with its own 10-bit mantissa.
//  - the weights are split and packed once (tf32_pack_kernel): chunk (tile
//    of 128 weight rows nt, K step of 32 ks) = the hi tile, then the lo
//    tile, each 16 KB in the UMMA K-major 128B-swizzle layout (row r, the 4
//    floats of group c at byte (r / 8) 1024 + (r % 8) 128 + ((c ^ (r % 8))
//    16)), zero past N and K;
//  - a CTA (256 threads) takes 128 rows of a by 128 weight rows over its K
//    range: the whole K, or with gridDim.z > 1 chunk z of KC, whose partial
//    (no bias) goes to y + z M N.  Per K step of 32 the weight chunk arrives
//    by one bulk copy, the threads load, split and store the a tile, and
//    thread 0 issues 4 x 3 MMAs (M 128, N 128, K 8); three stages: the
//    weight chunk of step j + 1 is requested at step j, and a step's loads
//    overlap the products of the steps before;
//  - the accumulator (TMEM lanes = rows of a, columns = weight rows) goes to
//    y by warps 0-7 (lane quarter warp % 4, column half warp / 4).
// An output element's sum runs over the same MMAs in the same order whatever
// M is, so frames decoded one call at a time still give the samples of one
// call.
constexpr int T3_ROWS = 128, T3_KS = 32;
constexpr int T3_TILE = T3_ROWS * T3_KS * 4;  // 16 KB
constexpr int T3_THREADS = 256;
constexpr int T3_STAGES = 3;
struct __align__(1024) T3Smem {
    uint8_t a[T3_STAGES][2][T3_TILE];  // [stage][hi, lo]
    uint8_t w[T3_STAGES][2][T3_TILE];  // [stage][hi, lo]: one packed chunk
    uint64_t wfull[T3_STAGES], mdone[T3_STAGES];
    uint32_t tmem_base;
};
static_assert(sizeof(T3Smem) + 1024 <= 232448, "codec products: shared memory above 227 KB");
static_assert(KC % T3_KS == 0, "a K chunk is whole K steps");
// c f32 (bit 4), a and b tf32 (2 at bits 7 and 10), K-major both, N 128, M 128
constexpr uint32_t T3_IDESC = (1u << 4) | (2u << 7) | (2u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);

__host__ __device__ inline uint32_t t3_off(int r, int c) {
    return (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4);
}
__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t u;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u) : "f"(x));
    return __uint_as_float(u);
}
__device__ __forceinline__ void t3_split_store(uint8_t *hi_tile, uint8_t *lo_tile, uint32_t off, const float *v) {
    float4 h, l;
    h.x = tf32_rna(v[0]);
    h.y = tf32_rna(v[1]);
    h.z = tf32_rna(v[2]);
    h.w = tf32_rna(v[3]);
    l.x = v[0] - h.x;
    l.y = v[1] - h.y;
    l.z = v[2] - h.z;
    l.w = v[3] - h.w;
    *reinterpret_cast<float4 *>(hi_tile + off) = h;
    *reinterpret_cast<float4 *>(lo_tile + off) = l;
}
__device__ __forceinline__ void umma_tf32(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(d),
        "l"(a), "l"(b), "r"(T3_IDESC), "r"(acc)
        : "memory");
}

// w [N][K] -> the packed chunks; one thread per (row of the padded tile
// grid, K step, group of 4)
__global__ void tf32_pack_kernel(const float *w, int N, int K, uint8_t *dst) {
    const int KS = (K + T3_KS - 1) / T3_KS, NT = (N + T3_ROWS - 1) / T3_ROWS;
    const long long total = static_cast<long long>(NT) * T3_ROWS * KS * (T3_KS / 4);
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % (T3_KS / 4));
        const long long rest = i / (T3_KS / 4);
        const int ks = static_cast<int>(rest % KS);
        const int row = static_cast<int>(rest / KS), nt = row / T3_ROWS, r = row % T3_ROWS;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int k = ks * T3_KS + 4 * c + j;
            v[j] = row < N && k < K ? w[static_cast<size_t>(row) * K + k] : 0.f;
        }
        uint8_t *chunk = dst + (static_cast<size_t>(nt) * KS + ks) * (2 * T3_TILE);
        t3_split_store(chunk, chunk + T3_TILE, t3_off(r, c), v);
    }
}

__global__ void __launch_bounds__(T3_THREADS, 1) tc3_gemm_kernel(const float *a, int M, int K, const uint8_t *wp,
                                                                int N, const float *bias, float *y, int *err) {
    extern __shared__ __align__(1024) uint8_t t3_raw[];
    T3Smem *sm = reinterpret_cast<T3Smem *>((reinterpret_cast<uintptr_t>(t3_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nt = blockIdx.x, m0 = blockIdx.y * T3_ROWS;
    const int KS = (K + T3_KS - 1) / T3_KS;
    const bool split = gridDim.z > 1;
    const int kb = split ? blockIdx.z * KC : 0, ke = split ? min(K, kb + KC) : K;
    const int s0 = kb / T3_KS, ns = (ke - kb + T3_KS - 1) / T3_KS;
    if (split) {
        y += static_cast<size_t>(blockIdx.z) * M * N;
        bias = nullptr;
    }
    if (tid == 0) {
        for (int b = 0; b < T3_STAGES; ++b) {
            qtts::mbar_init(&sm->wfull[b], 1);
            qtts::mbar_init(&sm->mdone[b], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {  // 128 f32 columns: the 128 x 128 accumulator
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;" ::"r"(
                         qtts::smem_u32(&sm->tmem_base))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tm = sm->tmem_base;
    // float4 loads where every row of a starts on 16 bytes
    const bool vec = (K & 3) == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0;
    bool good = true;
    int w_unwaited = -1;  // a step whose weight copy thread 0 gave up waiting for
    // step j's weight chunk goes to stage j % 3: the first three now, step
    // j + 1's at step j once the products of step j - 2 have freed its stage
    auto copy_w = [&](int j) {
        const int b = j % T3_STAGES;
        qtts::mbar_arrive_tx(&sm->wfull[b], 2 * T3_TILE);
        qtts::bulk_g2s(sm->w[b][0], wp + (static_cast<size_t>(nt) * KS + s0 + j) * (2 * T3_TILE), 2 * T3_TILE,
                       &sm->wfull[b]);
    };
    if (tid == 0)
        for (int j = 0; j < T3_STAGES && j < ns; ++j) copy_w(j);
    for (int i = 0; i < ns; ++i) {
        const int b = i % T3_STAGES, k0 = kb + T3_KS * i;
        const uint32_t par = (i / T3_STAGES) & 1;
        if (i >= 2) {
            // the products of step i - 2 are done: stage (i + 1) % 3 is free
            // for the a tile of step i + 1 and the weight chunk of step i + 1
            good = qtts::mbar_wait(&sm->mdone[(i - 2) % T3_STAGES], ((i - 2) / T3_STAGES) & 1, nullptr) && good;
            if (tid == 0 && i + 1 >= T3_STAGES && i + 1 < ns) copy_w(i + 1);
        }
        // a rows [m0, m0 + 128) x k [k0, k0 + 32): 1024 groups of 4, 4 per thread
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int g = tid + T3_THREADS * u, r = g >> 3, c = g & 7, m = m0 + r, k = k0 + 4 * c;
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (m < M) {
                const float *src = a + static_cast<size_t>(m) * K + k;
                if (vec) {
                    if (k < ke) {  // K % 4 == 0 and k0 % 4 == 0: the group is whole
                        const float4 q = *reinterpret_cast<const float4 *>(src);
                        v[0] = q.x;
                        v[1] = q.y;
                        v[2] = q.z;
                        v[3] = q.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) v[j] = k + j < ke ? src[j] : 0.f;
                }
            }
            t3_split_store(sm->a[b][0], sm->a[b][1], t3_off(r, c), v);
        }
        // the tensor core reads shared memory through the async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            if (qtts::mbar_wait(&sm->wfull[b], par, nullptr)) {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint64_t ah = qtts::umma_desc_sw128(sm->a[b][0]), al = qtts::umma_desc_sw128(sm->a[b][1]);
                const uint64_t wh = qtts::umma_desc_sw128(sm->w[b][0]), wl = qtts::umma_desc_sw128(sm->w[b][1]);
#pragma unroll
                for (int kk = 0; kk < T3_KS / 8; ++kk) {  // K 8 = 32 bytes = 2 units of 16 bytes
                    umma_tf32(tm, ah + 2 * kk, wh + 2 * kk, (i > 0 || kk > 0) ? 1u : 0u);
                    umma_tf32(tm, ah + 2 * kk, wl + 2 * kk, 1u);
                    umma_tf32(tm, al + 2 * kk, wh + 2 * kk, 1u);
                }
            } else {
                good = false;
                w_unwaited = i;
            }
            qtts::umma_commit(&sm->mdone[b]);  // also without products, so that the waits end
        }
    }
    // the last step's products, and with them every earlier one
    good = qtts::mbar_wait(&sm->mdone[(ns - 1) % T3_STAGES], ((ns - 1) / T3_STAGES) & 1, nullptr) && good;
    if (tid == 0 && w_unwaited >= 0)  // no copy may land after the CTA has gone
        qtts::mbar_wait(&sm->wfull[w_unwaited % T3_STAGES], (w_unwaited / T3_STAGES) & 1, nullptr);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    {
        const int q = warp & 3, half = warp >> 2, m = m0 + 32 * q + lane;
        for (int c = 64 * half; c < 64 * half + 64; c += 32) {
            float v[32];
            qtts::tmem_ld32(tm + (static_cast<uint32_t>(32 * q) << 16) + c, v);
            if (good && m < M) {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int n = nt * T3_ROWS + c + j;
                    if (n < N) y[static_cast<size_t>(m) * N + n] = v[j] + (bias ? bias[n] : 0.f);
                }
            }
        }
    }
    if (!good && err) atomicCAS(err, 0, QTTS_E_TIMEOUT);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;" ::"r"(tm) : "memory");
    }
}

// y[i] = (sum over z in order of part[z][i]) + bias[i % N]
__global__ void splitk_reduce_kernel(const float *part, int S, long long MN, int N, const float *bias, float *y) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < MN;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        float v = 0.f;
        for (int z = 0; z < S; ++z) v += part[static_cast<size_t>(z) * MN + i];
        y[i] = v + (bias ? bias[i % N] : 0.f);
    }
}

// col[r][c*K + k] = buf[r + k*dil][c]: the im2col rows of a causal
// convolution over [history ; input] (TQwenConv.Im2Col, codec.pas:317-334)
__global__ void im2col_kernel(const float *buf, int rows, int in, int K, int dil, float *col) {
    const long long n = static_cast<long long>(rows) * in * K;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(i / (static_cast<long long>(in) * K));
        const int rem = static_cast<int>(i - static_cast<long long>(r) * in * K);
        const int c = rem / K, k = rem - c * K;
        col[i] = buf[static_cast<size_t>(r + k * dil) * in + c];
    }
}

// x2[t][i*in + c] = buf[past + t - i][c] (TQwenTransConv.Forward, codec.pas:404-428)
__global__ void tgather_kernel(const float *buf, int rows, int in, int taps, float *x2) {
    const long long n = static_cast<long long>(rows) * taps * in;
    const int past = taps - 1;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int t = static_cast<int>(i / (static_cast<long long>(taps) * in));
        const int rem = static_cast<int>(i - static_cast<long long>(t) * taps * in);
        const int tap = rem / in, c = rem - tap * in;
        x2[i] = buf[static_cast<size_t>(past + t - tap) * in + c];
    }
}

// SnakeBeta in place (TQwenSnake.Apply, codec.pas:454-470)
__global__ void snake_kernel(float *x, long long n, int ch, const float *alpha, const float *inv_beta) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % ch);
        const float s = sinf(x[i] * alpha[c]);
        x[i] = x[i] + inv_beta[c] * (s * s);
    }
}

// the causal depthwise convolution of ConvNeXt (7 taps, codec.pas:514-523)
__global__ void dwconv_kernel(const float *buf, int rows, int dim, const float *w, const float *b, float *out) {
    const long long n = static_cast<long long>(rows) * dim;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int t = static_cast<int>(i / dim), c = static_cast<int>(i - static_cast<long long>(t) * dim);
        float acc = b[c];
        for (int k = 0; k < 7; ++k) acc += w[c * 7 + k] * buf[static_cast<size_t>(t + k) * dim + c];
        out[i] = acc;
    }
}

__device__ float block_sum(float v, float *red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    float s = 0.f;
    for (int i = 0; i < nw; ++i) s += red[i];
    return s;
}

// LayerNorm per row (eps 1e-6) in place, one block of 256 per row
__global__ void __launch_bounds__(256) layernorm_kernel(float *x, int dim, const float *w, const float *b) {
    __shared__ float red[8];
    float *r = x + static_cast<size_t>(blockIdx.x) * dim;
    float s = 0.f;
    for (int c = threadIdx.x; c < dim; c += blockDim.x) s += r[c];
    const float mean = block_sum(s, red) / static_cast<float>(dim);
    float v = 0.f;
    for (int c = threadIdx.x; c < dim; c += blockDim.x) v += (r[c] - mean) * (r[c] - mean);
    const float inv = 1.0f / sqrtf(block_sum(v, red) / static_cast<float>(dim) + 1e-6f);
    for (int c = threadIdx.x; c < dim; c += blockDim.x) r[c] = (r[c] - mean) * inv * w[c] + b[c];
}

// RMSNorm per row (eps 1e-5), one block of 256 per row
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float *x, int dim, const float *w, float *y) {
    __shared__ float red[8];
    const float *r = x + static_cast<size_t>(blockIdx.x) * dim;
    float s = 0.f;
    for (int c = threadIdx.x; c < dim; c += blockDim.x) s += r[c] * r[c];
    const float inv = 1.0f / sqrtf(block_sum(s, red) / static_cast<float>(dim) + 1e-5f);
    for (int c = threadIdx.x; c < dim; c += blockDim.x) y[static_cast<size_t>(blockIdx.x) * dim + c] = r[c] * inv * w[c];
}

__global__ void gelu_kernel(float *x, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        x[i] = 0.5f * x[i] * (1.0f + erff(x[i] * 0.70710678118654752f));
}

// y = x + scale[c] * v (ConvNeXt's gamma residual; the layer scales with y = x)
__global__ void scale_add_kernel(float *y, const float *x, const float *scale, const float *v, long long n, int dim) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        y[i] = x[i] + scale[i % dim] * v[i];
}

__global__ void add_kernel(float *y, const float *v, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        y[i] = v[i] + y[i];
}

__global__ void swiglu_kernel(float *g, const float *u, long long n) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        g[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
}

// rotate-half RoPE of rows x [rows][16 heads][64] with the angles' cos / sin
// [rows][32] (computed on the host in float32, as TQwenCodec.Transformer)
__global__ void rope_kernel(float *x, int rows, const float *cs, const float *sn) {
    const int n = rows * TF_HEADS * (TF_HD / 2);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int r = i / (TF_HEADS * (TF_HD / 2)), rem = i - r * (TF_HEADS * (TF_HD / 2));
        const int h = rem / (TF_HD / 2), j = rem - h * (TF_HD / 2);
        float *v = x + static_cast<size_t>(r) * TF_QKV + h * TF_HD;
        const float c = cs[r * (TF_HD / 2) + j], s = sn[r * (TF_HD / 2) + j];
        const float a = v[j], b = v[j + TF_HD / 2];
        v[j] = a * c - b * s;
        v[j + TF_HD / 2] = b * c + a * s;
    }
}

// sliding-window attention (codec.pas:990-1000): row r at position frames + r
// sees positions max(0, p - 71) .. p of the cache (rows from cache_base);
// one block of 128 per (row, head)
__global__ void __launch_bounds__(128) window_attn_kernel(const float *q, const float *keys, const float *values,
                                                          long long frames, long long cache_base, float *out) {
    __shared__ float sc[TF_WINDOW];
    __shared__ float red[4];
    const int r = blockIdx.x, h = blockIdx.y;
    const long long p = frames + r;
    long long first = p - (TF_WINDOW - 1);
    if (first < 0) first = 0;
    const int nk = static_cast<int>(p - first + 1);
    const float *qr = q + static_cast<size_t>(r) * TF_QKV + h * TF_HD;
    const size_t k0 = static_cast<size_t>(first - cache_base);
    float mx = -INFINITY;
    if (threadIdx.x < nk) {
        const float *kr = keys + (k0 + threadIdx.x) * TF_QKV + h * TF_HD;
        float s = 0.f;
        for (int d = 0; d < TF_HD; ++d) s = fmaf(qr[d], kr[d], s);
        s *= 0.125f;  // 1 / sqrt(64)
        sc[threadIdx.x] = s;
        mx = s;
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    float e = 0.f;
    if (threadIdx.x < nk) {
        e = expf(sc[threadIdx.x] - mx);
        sc[threadIdx.x] = e;
    }
    for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = e;
    __syncthreads();
    const float sum = red[0] + red[1] + red[2] + red[3];
    if (threadIdx.x < TF_HD) {
        float acc = 0.f;
        for (int j = 0; j < nk; ++j) acc += (sc[j] / sum) * values[(k0 + j) * TF_QKV + h * TF_HD + threadIdx.x];
        out[static_cast<size_t>(r) * TF_QKV + h * TF_HD + threadIdx.x] = acc;
    }
}

// the quantizer's sums (TQwenCodec.Quantize, codec.pas:886-917): q1 = the
// codebook 0 row, q2 = the rows of codebooks 1..15 added in order; codes
// checked on the host (negative ones read as 0)
__global__ void quant_kernel(const int *codes, const float *codebook, float *q1, float *q2) {
    const int f = blockIdx.x, c = threadIdx.x;  // CODE_DIM threads
    float s = 0.f;
    for (int g = 0; g < CG; ++g) {
        int code = codes[f * CG + g];
        code = code < 0 ? 0 : code;
        const float e = codebook[(static_cast<size_t>(g) * CB + code) * CODE_DIM + c];
        if (g == 0)
            q1[static_cast<size_t>(f) * CODE_DIM + c] = e;
        else
            s = g == 1 ? e : s + e;
    }
    q2[static_cast<size_t>(f) * CODE_DIM + c] = s;
}

__global__ void clamp_kernel(const float *a, long long n, float *pcm) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        pcm[i] = fminf(1.0f, fmaxf(-1.0f, a[i]));
}

inline unsigned blocks_for(long long n) {
    const long long b = (n + 255) / 256;
    return static_cast<unsigned>(b < 148 * 16 ? (b < 1 ? 1 : b) : 148 * 16);
}

}  // namespace qcodec

using namespace qcodec;

struct CConv {  // causal convolution: w [out][in*K] on the device, history rows
    int in, out, k, dil, past;
    float *w, *b, *hist;
};
struct CTConv {  // transposed convolution: w [s*out][taps*in], b [s*out]
    int in, out, s, taps;
    float *w, *b, *hist;
};
struct CSnake {
    int n;
    float *alpha, *inv_beta;
};
struct CNext {
    float *dw_w, *dw_b, *nw, *nb, *w1, *b1, *w2, *b2, *gamma, *hist;
};
struct CRes {
    CSnake a1, a2;
    CConv c1, c2;
    int dim;
};
struct CBlock {
    int in, out, rate;
    CSnake act;
    CTConv up;
    CRes res[3];
};
struct CTfLayer {
    float *in_norm, *wq, *wk, *wv, *wo, *post_norm, *wg, *wu, *wd, *attn_scale, *mlp_scale;
};

struct qtts_codec {
    qtts_device *dev;
    cudaStream_t st;
    std::vector<void *> allocs;
    float *codebook, *first_proj, *rest_proj;
    CConv pre;
    float *tf_in, *tf_in_b, *tf_out, *tf_out_b, *tf_norm;
    CTfLayer tf[TF_LAYERS];
    float *keys[TF_LAYERS] = {}, *values[TF_LAYERS] = {};
    int cache_cap = 0;
    long long cache_base = 0, frames = 0;
    float inv_freq[TF_HD / 2];
    CTConv up[2];
    CNext next[2];
    CConv conv0;
    CBlock blocks[4];
    CSnake act_out;
    CConv conv_out;
    // work buffers, grown on demand
    float *buf[13] = {};  // indexed by W_A .. W_PART
    size_t cap[13] = {};
    int *d_codes = nullptr;
    size_t codes_cap = 0;
    // the weights of the products, split and packed for tc3_gemm_kernel at
    // their first use (keyed by the float32 weights)
    std::unordered_map<const float *, const uint8_t *> packed;
    int *d_err = nullptr;  // error word of the bounded device waits
};

namespace {

enum { W_A, W_B, W_BUF, W_COL, W_X1, W_X2, W_T1, W_T2, W_T3, W_T4, W_T5, W_T6, W_PART };
static_assert(W_PART < 13, "qtts_codec::buf holds every work buffer");

int cx_scratch(qtts_codec *c, int i, size_t n, float **out) {
    if (c->cap[i] < n) {
        if (c->buf[i]) {
            CK(cudaStreamSynchronize(c->st));
            cudaFree(c->buf[i]);
        }
        c->buf[i] = nullptr;
        c->cap[i] = 0;
        if (cudaMalloc(&c->buf[i], n * 4) != cudaSuccess) return set_err(QTTS_E_OOM, "qtts_codec: out of device memory");
        c->cap[i] = n;
    }
    *out = c->buf[i];
    return QTTS_OK;
}

int cx_upload(qtts_codec *c, const float *h, size_t n, float **out) {
    *out = nullptr;
    if (cudaMalloc(out, n * 4) != cudaSuccess) return set_err(QTTS_E_OOM, "qtts_codec_create: out of device memory");
    c->allocs.push_back(*out);
    CK(cudaMemcpy(*out, h, n * 4, cudaMemcpyHostToDevice));
    return QTTS_OK;
}

// the tensor `name` of `count` values, widened to float32 on the host
// (F32 or BF16 in the file) and uploaded
int cx_tensor(qtts_codec *c, qtts_safetensors *f, const std::string &name, int64_t count, float **out) {
    std::vector<float> v;
    int rc = st_widen(f, name, count, v);
    if (rc) return rc;
    return cx_upload(c, v.data(), v.size(), out);
}

int cx_zeros(qtts_codec *c, size_t n, float **out) {
    *out = nullptr;
    if (cudaMalloc(out, (n ? n : 1) * 4) != cudaSuccess) return set_err(QTTS_E_OOM, "qtts_codec_create: out of device memory");
    c->allocs.push_back(*out);
    CK(cudaMemset(*out, 0, (n ? n : 1) * 4));
    return QTTS_OK;
}

int cx_conv(qtts_codec *c, qtts_safetensors *f, const std::string &p, int in, int out, int k, int dil, CConv &v) {
    v.in = in, v.out = out, v.k = k, v.dil = dil, v.past = (k - 1) * dil;
    int rc = cx_tensor(c, f, p + ".weight", static_cast<int64_t>(out) * in * k, &v.w);
    if (!rc) rc = cx_tensor(c, f, p + ".bias", out, &v.b);
    if (!rc) rc = cx_zeros(c, static_cast<size_t>(v.past) * in, &v.hist);
    return rc;
}

int cx_tconv(qtts_codec *c, qtts_safetensors *f, const std::string &p, int in, int out, int k, int s, CTConv &v) {
    v.in = in, v.out = out, v.s = s, v.taps = k / s;
    std::vector<float> w, b;
    int rc = st_widen(f, p + ".weight", static_cast<int64_t>(in) * out * k, w);
    if (!rc) rc = st_widen(f, p + ".bias", out, b);
    if (rc) return rc;
    const int cols = v.taps * in;
    std::vector<float> rw(static_cast<size_t>(s) * out * cols), rb(static_cast<size_t>(s) * out);
    for (int j = 0; j < s; ++j)
        for (int o = 0; o < out; ++o) {
            rb[static_cast<size_t>(j) * out + o] = b[o];
            for (int i = 0; i < v.taps; ++i)
                for (int ch = 0; ch < in; ++ch)
                    rw[(static_cast<size_t>(j) * out + o) * cols + i * in + ch] =
                        w[(static_cast<size_t>(ch) * out + o) * k + j + i * s];
        }
    rc = cx_upload(c, rw.data(), rw.size(), &v.w);
    if (!rc) rc = cx_upload(c, rb.data(), rb.size(), &v.b);
    if (!rc) rc = cx_zeros(c, static_cast<size_t>(v.taps - 1) * in, &v.hist);
    return rc;
}

// alpha = exp(a), inv_beta = 1 / (exp(b) + 1e-9), in float32 on the host
// (TQwenSnake.Create, codec.pas:431-452)
int cx_snake(qtts_codec *c, qtts_safetensors *f, const std::string &p, int n, CSnake &v) {
    v.n = n;
    std::vector<float> a, b;
    int rc = st_widen(f, p + ".alpha", n, a);
    if (!rc) rc = st_widen(f, p + ".beta", n, b);
    if (rc) return rc;
    for (int i = 0; i < n; ++i) {
        a[i] = expf(a[i]);
        b[i] = 1.0f / (expf(b[i]) + 1e-9f);
    }
    rc = cx_upload(c, a.data(), n, &v.alpha);
    if (!rc) rc = cx_upload(c, b.data(), n, &v.inv_beta);
    return rc;
}

void codec_free(qtts_codec *c) {
    for (void *p : c->allocs) cudaFree(p);
    for (int l = 0; l < TF_LAYERS; ++l) {
        if (c->keys[l]) cudaFree(c->keys[l]);
        if (c->values[l]) cudaFree(c->values[l]);
    }
    for (float *p : c->buf)
        if (p) cudaFree(p);
    if (c->d_codes) cudaFree(c->d_codes);
    if (c->d_err) cudaFree(c->d_err);
    if (c->st) cudaStreamDestroy(c->st);
    delete c;
}

// the split, tile-packed copy of w [N][K] (made on the stream at its first use)
int cx_packed(qtts_codec *c, const float *w, int N, int K, const uint8_t **out) {
    const auto it = c->packed.find(w);
    if (it != c->packed.end()) {
        *out = it->second;
        return QTTS_OK;
    }
    const size_t bytes = static_cast<size_t>((N + T3_ROWS - 1) / T3_ROWS) * ((K + T3_KS - 1) / T3_KS) * 2 * T3_TILE;
    uint8_t *p;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return set_err(QTTS_E_OOM, "qtts_codec: out of device memory");
    c->allocs.push_back(p);
    tf32_pack_kernel<<<blocks_for(static_cast<long long>(bytes / 32)), 256, 0, c->st>>>(w, N, K, p);
    CK(cudaGetLastError());
    c->packed[w] = p;
    *out = p;
    return QTTS_OK;
}

int cx_gemm(qtts_codec *c, const float *a, int M, int K, const float *w, int N, const float *bias, float *y) {
    if (M <= 0) return QTTS_OK;
    const uint8_t *wp;
    int rc = cx_packed(c, w, N, K, &wp);
    if (rc) return rc;
    const int S = (K + KC - 1) / KC;
    const size_t smem = sizeof(T3Smem) + 1024;
    if (S <= 1) {
        const dim3 grid((N + T3_ROWS - 1) / T3_ROWS, (M + T3_ROWS - 1) / T3_ROWS);
        qcodec::tc3_gemm_kernel<<<grid, T3_THREADS, smem, c->st>>>(a, M, K, wp, N, bias, y, c->d_err);
        CK(cudaGetLastError());
        return QTTS_OK;
    }
    // a long K: chunks of KC on their own CTAs, partials added in order
    float *part;
    const long long MN = static_cast<long long>(M) * N;
    rc = cx_scratch(c, W_PART, static_cast<size_t>(S) * MN, &part);
    if (rc) return rc;
    const dim3 grid((N + T3_ROWS - 1) / T3_ROWS, (M + T3_ROWS - 1) / T3_ROWS, S);
    qcodec::tc3_gemm_kernel<<<grid, T3_THREADS, smem, c->st>>>(a, M, K, wp, N, nullptr, part, c->d_err);
    CK(cudaGetLastError());
    qcodec::splitk_reduce_kernel<<<blocks_for(MN), 256, 0, c->st>>>(part, S, MN, N, bias, y);
    CK(cudaGetLastError());
    return QTTS_OK;
}

// y[rows][out] = the causal convolution of x[rows][in] (TQwenConv.Forward)
int cx_conv_fwd(qtts_codec *c, CConv &v, const float *x, int rows, float *y) {
    if (v.k == 1) return cx_gemm(c, x, rows, v.in, v.w, v.out, v.b, y);
    float *buf, *col;
    const size_t nb = static_cast<size_t>(v.past + rows) * v.in, nc = static_cast<size_t>(rows) * v.in * v.k;
    int rc = cx_scratch(c, W_BUF, nb, &buf);
    if (!rc) rc = cx_scratch(c, W_COL, nc, &col);
    if (rc) return rc;
    CK(cudaMemcpyAsync(buf, v.hist, static_cast<size_t>(v.past) * v.in * 4, cudaMemcpyDeviceToDevice, c->st));
    CK(cudaMemcpyAsync(buf + static_cast<size_t>(v.past) * v.in, x, static_cast<size_t>(rows) * v.in * 4,
                       cudaMemcpyDeviceToDevice, c->st));
    im2col_kernel<<<blocks_for(static_cast<long long>(nc)), 256, 0, c->st>>>(buf, rows, v.in, v.k, v.dil, col);
    CK(cudaGetLastError());
    rc = cx_gemm(c, col, rows, v.in * v.k, v.w, v.out, v.b, y);
    if (rc) return rc;
    CK(cudaMemcpyAsync(v.hist, buf + static_cast<size_t>(rows) * v.in, static_cast<size_t>(v.past) * v.in * 4,
                       cudaMemcpyDeviceToDevice, c->st));
    return QTTS_OK;
}

// y[rows * s][out] (TQwenTransConv.Forward)
int cx_tconv_fwd(qtts_codec *c, CTConv &v, const float *x, int rows, float *y) {
    if (v.taps == 1) return cx_gemm(c, x, rows, v.in, v.w, v.s * v.out, v.b, y);
    const int past = v.taps - 1;
    float *buf, *x2;
    const size_t nb = static_cast<size_t>(past + rows) * v.in, n2 = static_cast<size_t>(rows) * v.taps * v.in;
    int rc = cx_scratch(c, W_BUF, nb, &buf);
    if (!rc) rc = cx_scratch(c, W_COL, n2, &x2);
    if (rc) return rc;
    CK(cudaMemcpyAsync(buf, v.hist, static_cast<size_t>(past) * v.in * 4, cudaMemcpyDeviceToDevice, c->st));
    CK(cudaMemcpyAsync(buf + static_cast<size_t>(past) * v.in, x, static_cast<size_t>(rows) * v.in * 4,
                       cudaMemcpyDeviceToDevice, c->st));
    tgather_kernel<<<blocks_for(static_cast<long long>(n2)), 256, 0, c->st>>>(buf, rows, v.in, v.taps, x2);
    CK(cudaGetLastError());
    rc = cx_gemm(c, x2, rows, v.taps * v.in, v.w, v.s * v.out, v.b, y);
    if (rc) return rc;
    CK(cudaMemcpyAsync(v.hist, buf + static_cast<size_t>(rows) * v.in, static_cast<size_t>(past) * v.in * 4,
                       cudaMemcpyDeviceToDevice, c->st));
    return QTTS_OK;
}

int cx_snake_fwd(qtts_codec *c, const CSnake &s, float *x, int rows) {
    const long long n = static_cast<long long>(rows) * s.n;
    snake_kernel<<<blocks_for(n), 256, 0, c->st>>>(x, n, s.n, s.alpha, s.inv_beta);
    CK(cudaGetLastError());
    return QTTS_OK;
}

// y = x + ConvNeXt(x), rows of LATENT (TQwenConvNeXt.Forward)
int cx_next_fwd(qtts_codec *c, CNext &v, const float *x, int rows, float *y) {
    const int D = LATENT;
    float *buf, *n, *h;
    int rc = cx_scratch(c, W_BUF, static_cast<size_t>(6 + rows) * D, &buf);
    if (!rc) rc = cx_scratch(c, W_T1, static_cast<size_t>(rows) * D, &n);
    if (!rc) rc = cx_scratch(c, W_T2, static_cast<size_t>(rows) * 4 * D, &h);
    if (rc) return rc;
    CK(cudaMemcpyAsync(buf, v.hist, static_cast<size_t>(6) * D * 4, cudaMemcpyDeviceToDevice, c->st));
    CK(cudaMemcpyAsync(buf + static_cast<size_t>(6) * D, x, static_cast<size_t>(rows) * D * 4, cudaMemcpyDeviceToDevice,
                       c->st));
    dwconv_kernel<<<blocks_for(static_cast<long long>(rows) * D), 256, 0, c->st>>>(buf, rows, D, v.dw_w, v.dw_b, n);
    CK(cudaMemcpyAsync(v.hist, buf + static_cast<size_t>(rows) * D, static_cast<size_t>(6) * D * 4,
                       cudaMemcpyDeviceToDevice, c->st));
    layernorm_kernel<<<rows, 256, 0, c->st>>>(n, D, v.nw, v.nb);
    CK(cudaGetLastError());
    if ((rc = cx_gemm(c, n, rows, D, v.w1, 4 * D, v.b1, h))) return rc;
    gelu_kernel<<<blocks_for(static_cast<long long>(rows) * 4 * D), 256, 0, c->st>>>(h, static_cast<long long>(rows) * 4 * D);
    if ((rc = cx_gemm(c, h, rows, 4 * D, v.w2, D, v.b2, n))) return rc;
    scale_add_kernel<<<blocks_for(static_cast<long long>(rows) * D), 256, 0, c->st>>>(
        y, x, v.gamma, n, static_cast<long long>(rows) * D, D);
    CK(cudaGetLastError());
    return QTTS_OK;
}

// the cache keeps positions cache_base .. frames-1 (TQwenCodec.CacheRoom)
int cx_cache_room(qtts_codec *c, int rows) {
    if (c->frames - c->cache_base + rows <= c->cache_cap) return QTTS_OK;
    long long keep = c->frames - c->cache_base;
    if (keep > TF_WINDOW - 1) keep = TF_WINDOW - 1;
    const long long from = c->frames - c->cache_base - keep;
    const size_t kb = static_cast<size_t>(keep) * TF_QKV * 4;
    if (keep + rows > c->cache_cap) {
        const int cap = static_cast<int>(keep) + rows + 4 * TF_WINDOW;
        CK(cudaStreamSynchronize(c->st));
        for (int l = 0; l < TF_LAYERS; ++l) {
            float *k = nullptr, *v = nullptr;
            if (cudaMalloc(&k, static_cast<size_t>(cap) * TF_QKV * 4) != cudaSuccess ||
                cudaMalloc(&v, static_cast<size_t>(cap) * TF_QKV * 4) != cudaSuccess) {
                if (k) cudaFree(k);
                return set_err(QTTS_E_OOM, "qtts_codec_decode: out of device memory");
            }
            if (keep > 0 && c->keys[l]) {
                CK(cudaMemcpy(k, c->keys[l] + from * TF_QKV, kb, cudaMemcpyDeviceToDevice));
                CK(cudaMemcpy(v, c->values[l] + from * TF_QKV, kb, cudaMemcpyDeviceToDevice));
            }
            if (c->keys[l]) cudaFree(c->keys[l]);
            if (c->values[l]) cudaFree(c->values[l]);
            c->keys[l] = k, c->values[l] = v;
        }
        c->cache_cap = cap;
    } else if (keep > 0 && from > 0) {
        // the kept rows to the front, through a work buffer (the ranges may overlap)
        float *tmp;
        int rc = cx_scratch(c, W_T6, static_cast<size_t>(keep) * TF_QKV, &tmp);
        if (rc) return rc;
        for (int l = 0; l < TF_LAYERS; ++l)
            for (float *p : {c->keys[l], c->values[l]}) {
                CK(cudaMemcpyAsync(tmp, p + from * TF_QKV, kb, cudaMemcpyDeviceToDevice, c->st));
                CK(cudaMemcpyAsync(p, tmp, kb, cudaMemcpyDeviceToDevice, c->st));
            }
    }
    c->cache_base = c->frames - keep;
    return QTTS_OK;
}

// TQwenCodec.Transformer (codec.pas:948-1017): x [rows][LATENT] -> y
int cx_transformer(qtts_codec *c, const float *x, int rows, float *y) {
    const size_t R = static_cast<size_t>(rows);
    float *h, *n, *q, *k, *v, *att, *o, *g, *u;
    int rc;
    if ((rc = cx_scratch(c, W_T1, R * TF_DIM, &h)) || (rc = cx_scratch(c, W_T2, R * TF_DIM, &n)) ||
        (rc = cx_scratch(c, W_T3, R * TF_QKV * 3, &q)) || (rc = cx_scratch(c, W_T4, R * TF_QKV, &att)) ||
        (rc = cx_scratch(c, W_T5, R * (TF_DIM + 2 * TF_MLP), &o)))
        return rc;
    k = q + R * TF_QKV;
    v = k + R * TF_QKV;
    g = o + R * TF_DIM;
    u = g + R * TF_MLP;
    // RoPE angles: (frames + r) * inv_freq_i in float32, cos / sin
    std::vector<float> cs(R * (TF_HD / 2) * 2);
    for (size_t r = 0; r < R; ++r)
        for (int i = 0; i < TF_HD / 2; ++i) {
            const float a = static_cast<float>(c->frames + static_cast<long long>(r)) * c->inv_freq[i];
            cs[r * (TF_HD / 2) + i] = cosf(a);
            cs[(R + r) * (TF_HD / 2) + i] = sinf(a);
        }
    float *d_cs;
    if ((rc = cx_scratch(c, W_X2, cs.size(), &d_cs))) return rc;
    CK(cudaMemcpyAsync(d_cs, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, c->st));
    CK(cudaStreamSynchronize(c->st));  // cs is a host vector of this call
    if ((rc = cx_gemm(c, x, rows, LATENT, c->tf_in, TF_DIM, c->tf_in_b, h))) return rc;
    if ((rc = cx_cache_room(c, rows))) return rc;
    const long long row0 = c->frames - c->cache_base;
    const unsigned nb = blocks_for(static_cast<long long>(rows) * TF_HEADS * (TF_HD / 2));
    for (int l = 0; l < TF_LAYERS; ++l) {
        CTfLayer &w = c->tf[l];
        rmsnorm_kernel<<<rows, 256, 0, c->st>>>(h, TF_DIM, w.in_norm, n);
        if ((rc = cx_gemm(c, n, rows, TF_DIM, w.wq, TF_QKV, nullptr, q)) ||
            (rc = cx_gemm(c, n, rows, TF_DIM, w.wk, TF_QKV, nullptr, k)) ||
            (rc = cx_gemm(c, n, rows, TF_DIM, w.wv, TF_QKV, nullptr, v)))
            return rc;
        rope_kernel<<<nb, 256, 0, c->st>>>(q, rows, d_cs, d_cs + R * (TF_HD / 2));
        rope_kernel<<<nb, 256, 0, c->st>>>(k, rows, d_cs, d_cs + R * (TF_HD / 2));
        CK(cudaMemcpyAsync(c->keys[l] + row0 * TF_QKV, k, R * TF_QKV * 4, cudaMemcpyDeviceToDevice, c->st));
        CK(cudaMemcpyAsync(c->values[l] + row0 * TF_QKV, v, R * TF_QKV * 4, cudaMemcpyDeviceToDevice, c->st));
        window_attn_kernel<<<dim3(rows, TF_HEADS), 128, 0, c->st>>>(q, c->keys[l], c->values[l], c->frames,
                                                                     c->cache_base, att);
        CK(cudaGetLastError());
        if ((rc = cx_gemm(c, att, rows, TF_QKV, w.wo, TF_DIM, nullptr, o))) return rc;
        scale_add_kernel<<<blocks_for(R * TF_DIM), 256, 0, c->st>>>(h, h, w.attn_scale, o, R * TF_DIM, TF_DIM);
        rmsnorm_kernel<<<rows, 256, 0, c->st>>>(h, TF_DIM, w.post_norm, n);
        if ((rc = cx_gemm(c, n, rows, TF_DIM, w.wg, TF_MLP, nullptr, g)) ||
            (rc = cx_gemm(c, n, rows, TF_DIM, w.wu, TF_MLP, nullptr, u)))
            return rc;
        swiglu_kernel<<<blocks_for(R * TF_MLP), 256, 0, c->st>>>(g, u, R * TF_MLP);
        if ((rc = cx_gemm(c, g, rows, TF_MLP, w.wd, TF_DIM, nullptr, o))) return rc;
        scale_add_kernel<<<blocks_for(R * TF_DIM), 256, 0, c->st>>>(h, h, w.mlp_scale, o, R * TF_DIM, TF_DIM);
        CK(cudaGetLastError());
    }
    rmsnorm_kernel<<<rows, 256, 0, c->st>>>(h, TF_DIM, c->tf_norm, n);
    CK(cudaGetLastError());
    return cx_gemm(c, n, rows, TF_DIM, c->tf_out, LATENT, c->tf_out_b, y);
}

}  // namespace

extern "C" int qtts_codec_destroy(qtts_codec *c) {
    if (!c) return QTTS_OK;
    cudaSetDevice(c->dev->ordinal);
    codec_free(c);
    return QTTS_OK;
}

extern "C" int qtts_codec_create_safetensors(qtts_device *dev, qtts_safetensors *f, qtts_codec **out) {
    if (!dev || !f || !out) return set_err(QTTS_E_ARG, "qtts_codec_create_safetensors: NULL argument");
    *out = nullptr;
    CK(cudaSetDevice(dev->ordinal));
    qtts_codec *c = new qtts_codec();
    c->dev = dev;
    if (cudaStreamCreateWithFlags(&c->st, cudaStreamNonBlocking) != cudaSuccess) {
        c->st = nullptr;
        codec_free(c);
        return set_err(QTTS_E_CUDA, "qtts_codec_create_safetensors: no stream");
    }
    if (cudaMalloc(&c->d_err, 4) != cudaSuccess || cudaMemsetAsync(c->d_err, 0, 4, c->st) != cudaSuccess ||
        cudaFuncSetAttribute(tc3_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sizeof(T3Smem) + 1024)) != cudaSuccess) {
        codec_free(c);
        return set_err(QTTS_E_CUDA, "qtts_codec_create_safetensors: device setup failed");
    }
    int rc = QTTS_OK;
    // the quantizer: codebook = embedding_sum / max(cluster_usage, 1e-5)
    {
        std::vector<float> cb(static_cast<size_t>(CG) * CB * CODE_DIM), sum, use;
        for (int g = 0; g < CG && !rc; ++g) {
            const std::string p = g == 0 ? std::string("decoder.quantizer.rvq_first.vq.layers.0._codebook")
                                         : "decoder.quantizer.rvq_rest.vq.layers." + std::to_string(g - 1) + "._codebook";
            rc = st_widen(f, p + ".embedding_sum", static_cast<int64_t>(CB) * CODE_DIM, sum);
            if (!rc) rc = st_widen(f, p + ".cluster_usage", CB, use);
            if (rc) break;
            for (int i = 0; i < CB; ++i) {
                const float d = use[i] < 1e-5f ? 1e-5f : use[i];
                for (int ch = 0; ch < CODE_DIM; ++ch)
                    cb[(static_cast<size_t>(g) * CB + i) * CODE_DIM + ch] = sum[static_cast<size_t>(i) * CODE_DIM + ch] / d;
            }
        }
        if (!rc) rc = cx_upload(c, cb.data(), cb.size(), &c->codebook);
    }
    if (!rc) rc = cx_tensor(c, f, "decoder.quantizer.rvq_first.output_proj.weight", QUANT_DIM * CODE_DIM, &c->first_proj);
    if (!rc) rc = cx_tensor(c, f, "decoder.quantizer.rvq_rest.output_proj.weight", QUANT_DIM * CODE_DIM, &c->rest_proj);
    if (!rc) rc = cx_conv(c, f, "decoder.pre_conv.conv", QUANT_DIM, LATENT, 3, 1, c->pre);
    const std::string tp = "decoder.pre_transformer.";
    if (!rc) rc = cx_tensor(c, f, tp + "input_proj.weight", TF_DIM * LATENT, &c->tf_in);
    if (!rc) rc = cx_tensor(c, f, tp + "input_proj.bias", TF_DIM, &c->tf_in_b);
    if (!rc) rc = cx_tensor(c, f, tp + "output_proj.weight", LATENT * TF_DIM, &c->tf_out);
    if (!rc) rc = cx_tensor(c, f, tp + "output_proj.bias", LATENT, &c->tf_out_b);
    if (!rc) rc = cx_tensor(c, f, tp + "norm.weight", TF_DIM, &c->tf_norm);
    for (int l = 0; l < TF_LAYERS && !rc; ++l) {
        const std::string p = tp + "layers." + std::to_string(l) + ".";
        CTfLayer &w = c->tf[l];
        struct {
            const char *n;
            int64_t count;
            float **dst;
        } t[] = {{"input_layernorm.weight", TF_DIM, &w.in_norm},
                 {"self_attn.q_proj.weight", static_cast<int64_t>(TF_QKV) * TF_DIM, &w.wq},
                 {"self_attn.k_proj.weight", static_cast<int64_t>(TF_QKV) * TF_DIM, &w.wk},
                 {"self_attn.v_proj.weight", static_cast<int64_t>(TF_QKV) * TF_DIM, &w.wv},
                 {"self_attn.o_proj.weight", static_cast<int64_t>(TF_DIM) * TF_QKV, &w.wo},
                 {"post_attention_layernorm.weight", TF_DIM, &w.post_norm},
                 {"mlp.gate_proj.weight", static_cast<int64_t>(TF_MLP) * TF_DIM, &w.wg},
                 {"mlp.up_proj.weight", static_cast<int64_t>(TF_MLP) * TF_DIM, &w.wu},
                 {"mlp.down_proj.weight", static_cast<int64_t>(TF_DIM) * TF_MLP, &w.wd},
                 {"self_attn_layer_scale.scale", TF_DIM, &w.attn_scale},
                 {"mlp_layer_scale.scale", TF_DIM, &w.mlp_scale}};
        for (auto &e : t)
            if (!rc) rc = cx_tensor(c, f, p + e.n, e.count, e.dst);
    }
    // RoPE base 10000: inv_freq_i = 1 / 10000^(2i/64), rounded to float32
    for (int i = 0; i < TF_HD / 2; ++i)
        c->inv_freq[i] = static_cast<float>(1.0 / exp(log(10000.0) * (2.0 * i / TF_HD)));
    for (int i = 0; i < 2 && !rc; ++i) {
        const std::string p = "decoder.upsample." + std::to_string(i);
        rc = cx_tconv(c, f, p + ".0.conv", LATENT, LATENT, 2, 2, c->up[i]);
        CNext &x = c->next[i];
        const std::string q = p + ".1.";
        if (!rc) rc = cx_tensor(c, f, q + "dwconv.conv.weight", LATENT * 7, &x.dw_w);
        if (!rc) rc = cx_tensor(c, f, q + "dwconv.conv.bias", LATENT, &x.dw_b);
        if (!rc) rc = cx_tensor(c, f, q + "norm.weight", LATENT, &x.nw);
        if (!rc) rc = cx_tensor(c, f, q + "norm.bias", LATENT, &x.nb);
        if (!rc) rc = cx_tensor(c, f, q + "pwconv1.weight", static_cast<int64_t>(4) * LATENT * LATENT, &x.w1);
        if (!rc) rc = cx_tensor(c, f, q + "pwconv1.bias", 4 * LATENT, &x.b1);
        if (!rc) rc = cx_tensor(c, f, q + "pwconv2.weight", static_cast<int64_t>(4) * LATENT * LATENT, &x.w2);
        if (!rc) rc = cx_tensor(c, f, q + "pwconv2.bias", LATENT, &x.b2);
        if (!rc) rc = cx_tensor(c, f, q + "gamma", LATENT, &x.gamma);
        if (!rc) rc = cx_zeros(c, static_cast<size_t>(6) * LATENT, &x.hist);
    }
    if (!rc) rc = cx_conv(c, f, "decoder.decoder.0.conv", LATENT, DEC_DIM, 7, 1, c->conv0);
    static const int rates[4] = {8, 5, 4, 3}, dil[3] = {1, 3, 9};
    for (int b = 0; b < 4 && !rc; ++b) {
        CBlock &k = c->blocks[b];
        k.in = DEC_DIM >> b, k.out = DEC_DIM >> (b + 1), k.rate = rates[b];
        const std::string p = "decoder.decoder." + std::to_string(b + 1) + ".block.";
        rc = cx_snake(c, f, p + "0", k.in, k.act);
        if (!rc) rc = cx_tconv(c, f, p + "1.conv", k.in, k.out, 2 * k.rate, k.rate, k.up);
        for (int r = 0; r < 3 && !rc; ++r) {
            CRes &u = k.res[r];
            u.dim = k.out;
            const std::string q = p + std::to_string(r + 2) + ".";
            rc = cx_snake(c, f, q + "act1", k.out, u.a1);
            if (!rc) rc = cx_conv(c, f, q + "conv1.conv", k.out, k.out, 7, dil[r], u.c1);
            if (!rc) rc = cx_snake(c, f, q + "act2", k.out, u.a2);
            if (!rc) rc = cx_conv(c, f, q + "conv2.conv", k.out, k.out, 1, 1, u.c2);
        }
    }
    if (!rc) rc = cx_snake(c, f, "decoder.decoder.5", DEC_DIM >> 4, c->act_out);
    if (!rc) rc = cx_conv(c, f, "decoder.decoder.6.conv", DEC_DIM >> 4, 1, 7, 1, c->conv_out);
    if (rc) {
        codec_free(c);
        return rc;
    }
    *out = c;
    return QTTS_OK;
}

extern "C" int qtts_codec_reset(qtts_codec *c) {
    if (!c) return set_err(QTTS_E_ARG, "qtts_codec_reset: NULL codec");
    CK(cudaSetDevice(c->dev->ordinal));
    c->frames = 0;
    c->cache_base = 0;
    auto zero = [c](float *p, size_t n) -> int {
        if (n) CK(cudaMemsetAsync(p, 0, n * 4, c->st));
        return QTTS_OK;
    };
    int rc = zero(c->pre.hist, static_cast<size_t>(c->pre.past) * c->pre.in);
    for (int i = 0; i < 2; ++i) {
        rc |= zero(c->up[i].hist, static_cast<size_t>(c->up[i].taps - 1) * c->up[i].in);
        rc |= zero(c->next[i].hist, static_cast<size_t>(6) * LATENT);
    }
    rc |= zero(c->conv0.hist, static_cast<size_t>(c->conv0.past) * c->conv0.in);
    for (int b = 0; b < 4; ++b) {
        CBlock &k = c->blocks[b];
        rc |= zero(k.up.hist, static_cast<size_t>(k.up.taps - 1) * k.up.in);
        for (int r = 0; r < 3; ++r) rc |= zero(k.res[r].c1.hist, static_cast<size_t>(k.res[r].c1.past) * k.res[r].c1.in);
    }
    rc |= zero(c->conv_out.hist, static_cast<size_t>(c->conv_out.past) * c->conv_out.in);
    if (rc) return QTTS_E_CUDA;
    CK(cudaStreamSynchronize(c->st));
    return QTTS_OK;
}

extern "C" int qtts_codec_frames(qtts_codec *c, int64_t *frames) {
    if (!c || !frames) return set_err(QTTS_E_ARG, "qtts_codec_frames: bad argument");
    *frames = c->frames;
    return QTTS_OK;
}

extern "C" int qtts_codec_decode(qtts_codec *c, const int32_t *codes, int frames, float *pcm) {
    if (!c || (frames > 0 && (!codes || !pcm))) return set_err(QTTS_E_ARG, "qtts_codec_decode: NULL argument");
    if (frames <= 0) return QTTS_OK;
    // at most 2048 frames a call: the GEMM grid's rows (1920 per frame / 64)
    // stay within its 65535 limit
    if (frames > 2048) return set_err(QTTS_E_ARG, "qtts_codec_decode: %d frames in one call (at most 2048)", frames);
    for (int i = 0; i < frames * CG; ++i)
        if (codes[i] >= CB)
            return set_err(QTTS_E_ARG, "qtts_codec_decode: code %d out of range in group %d", codes[i], i % CG);
    CK(cudaSetDevice(c->dev->ordinal));
    const size_t F = static_cast<size_t>(frames);
    const size_t big = std::max(F * FRAME_SAMPLES * (DEC_DIM >> 4), F * 4 * DEC_DIM);
    float *a, *b, *x1, *x2;
    int rc;
    if ((rc = cx_scratch(c, W_A, big, &a)) || (rc = cx_scratch(c, W_B, big, &b)) || (rc = cx_scratch(c, W_X1, big, &x1)))
        return rc;
    if (F * CG > c->codes_cap) {
        if (c->d_codes) {
            CK(cudaStreamSynchronize(c->st));
            cudaFree(c->d_codes);
        }
        c->d_codes = nullptr;
        c->codes_cap = 0;
        if (cudaMalloc(&c->d_codes, F * CG * 4) != cudaSuccess) return set_err(QTTS_E_OOM, "qtts_codec_decode: out of device memory");
        c->codes_cap = F * CG;
    }
    CK(cudaMemcpyAsync(c->d_codes, codes, F * CG * 4, cudaMemcpyHostToDevice, c->st));
    CK(cudaStreamSynchronize(c->st));  // codes is the caller's pageable buffer
    // the quantizer: q1 in x1, q2 after it; the two projections into a and b
    float *q1 = x1, *q2 = x1 + F * CODE_DIM;
    quant_kernel<<<frames, CODE_DIM, 0, c->st>>>(c->d_codes, c->codebook, q1, q2);
    CK(cudaGetLastError());
    if ((rc = cx_gemm(c, q1, frames, CODE_DIM, c->first_proj, QUANT_DIM, nullptr, a)) ||
        (rc = cx_gemm(c, q2, frames, CODE_DIM, c->rest_proj, QUANT_DIM, nullptr, b)))
        return rc;
    add_kernel<<<blocks_for(static_cast<long long>(F) * QUANT_DIM), 256, 0, c->st>>>(a, b, static_cast<long long>(F) * QUANT_DIM);
    if ((rc = cx_conv_fwd(c, c->pre, a, frames, b))) return rc;
    if ((rc = cx_transformer(c, b, frames, a))) return rc;
    // the back part (TQwenCodec.Back, codec.pas:1040-1084)
    int rows = frames;
    for (int i = 0; i < 2; ++i) {
        if ((rc = cx_tconv_fwd(c, c->up[i], a, rows, b))) return rc;
        rows *= 2;
        if ((rc = cx_next_fwd(c, c->next[i], b, rows, a))) return rc;
    }
    if ((rc = cx_conv_fwd(c, c->conv0, a, rows, b))) return rc;
    for (int k = 0; k < 4; ++k) {
        CBlock &bl = c->blocks[k];
        if ((rc = cx_snake_fwd(c, bl.act, b, rows))) return rc;
        if ((rc = cx_tconv_fwd(c, bl.up, b, rows, a))) return rc;
        rows *= bl.rate;
        for (int r = 0; r < 3; ++r) {
            CRes &u = bl.res[r];
            const long long n = static_cast<long long>(rows) * u.dim;
            if ((rc = cx_scratch(c, W_X2, static_cast<size_t>(n), &x2))) return rc;
            CK(cudaMemcpyAsync(x1, a, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToDevice, c->st));
            if ((rc = cx_snake_fwd(c, u.a1, x1, rows)) || (rc = cx_conv_fwd(c, u.c1, x1, rows, x2)) ||
                (rc = cx_snake_fwd(c, u.a2, x2, rows)) || (rc = cx_conv_fwd(c, u.c2, x2, rows, x1)))
                return rc;
            add_kernel<<<blocks_for(n), 256, 0, c->st>>>(a, x1, n);
            CK(cudaGetLastError());
        }
        std::swap(a, b);
    }
    if ((rc = cx_snake_fwd(c, c->act_out, b, rows)) || (rc = cx_conv_fwd(c, c->conv_out, b, rows, a))) return rc;
    clamp_kernel<<<blocks_for(rows), 256, 0, c->st>>>(a, rows, a);
    CK(cudaGetLastError());
    CK(cudaMemcpyAsync(pcm, a, static_cast<size_t>(rows) * 4, cudaMemcpyDeviceToHost, c->st));
    int h_err = 0;
    CK(cudaMemcpyAsync(&h_err, c->d_err, 4, cudaMemcpyDeviceToHost, c->st));
    CK(cudaStreamSynchronize(c->st));
    if (h_err) {
        CK(cudaMemsetAsync(c->d_err, 0, 4, c->st));
        CK(cudaStreamSynchronize(c->st));
        return set_err(QTTS_E_TIMEOUT, "qtts_codec_decode: a device wait gave up");
    }
    c->frames += frames;
    return QTTS_OK;
}
