// qtts_api.cu -- the C-ABI of libqtts.so (declared in include/qtts.h).
//
// Host side of the B200 implementation of mormot2-qwen-tts's per-frame
// language-model path.  Handles mirror the reference's objects:
//   qtts_stack  ~ TDecoderModel from QwenLmStack (mormot.ai.tts.qwen.lm.pas:174-179)
//   qtts_heads  ~ TQwenLmHeads (lm.pas:64-100, 225-332)
//   qtts_lm     ~ TQwenLm (lm.pas:102-143, 335-408)
//   qtts_talker ~ the per-frame part of TQwenTalker (mormot.ai.tts.qwen.talker.pas:595-681)
//   qtts_batch / qtts_talkers ~ the same protocols for many utterances at once
// Batch 1 runs in the persistent kernel of qtts_decode.cuh, batches on the
// tcgen05 GEMM (qtts_gemm.cuh) and the kernels of qtts_batch.cuh; this file
// uploads and packs weights (bit-exact ggml Q8_0 quantisation on the
// device), owns the device memory, launches and captures the frame graphs.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/qtts.h"
#include "qtts_decode.cuh"
#include "qtts_gemm.cuh"
#include "qtts_batch.cuh"
#include "qtts_safetensors.h"

#include <cudaTypedefs.h>

using namespace qtts;

// ------------------------------------------------------------------ errors

static thread_local std::string g_err;

static int set_err(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CK(call)                                                                                     \
    do {                                                                                             \
        cudaError_t e_ = (call);                                                                     \
        if (e_ != cudaSuccess) {                                                                     \
            int c_ = (e_ == cudaErrorMemoryAllocation) ? QTTS_E_OOM : QTTS_E_CUDA;                   \
            return set_err(c_, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
        }                                                                                            \
    } while (0)

extern "C" const char *qtts_last_error(void) { return g_err.c_str(); }

// ------------------------------------------------------------------ launches

// a kernel launch with programmatic stream serialisation: the kernel may
// start while its predecessor on the stream runs (its pdl_wait() orders the
// dependent work), which hides launch and prologue latency between the
// short kernels of the batched path, in graphs too
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// the same with thread-block clusters of cluster_z CTAs along z (> 1)
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                      unsigned cluster_z, Args &&...args) {
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = cluster_z;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------ handles

struct qtts_device {
    int ordinal;
    int sms;
    size_t smem;
    cudaStream_t load;  // uploads
    void *staging;      // device staging for uploads
    size_t staging_bytes;
    int64_t bytes;      // stack weights held (TQwenVulkan.DeviceBytes)
    char name[256];
    float *draw_in;     // qtts_sample: SAMPLE_MAX_V values + the code (made on first use)
};

struct qtts_stack {
    qtts_device *dev;
    qtts_stack_config cfg;
    std::vector<void *> allocs;
    std::vector<DLayer> hlayers;  // the same table, host side
    std::vector<DLayer> tlayers;  // the matrices tile-packed for the GEMM (built on first batched use)
    DLayer *d_layers;
    float *d_final_norm;
    int64_t bytes;
    int keep_l2;
};

struct HeadMat {
    uint8_t *d;
    int rows;
    uint8_t *t;  // tile-packed for the GEMM (built on first use), or NULL
};

struct qtts_heads {
    qtts_device *dev;
    std::string name;
    int hidden, dtype;
    std::vector<HeadMat> mats;
    int64_t bytes;
    // buffers of qtts_heads_linear (grown on demand)
    float *lx = nullptr, *ly = nullptr;
    __half *lh = nullptr;
    int *lerr = nullptr;
    size_t lrows = 0, lycap = 0;
};

struct Runner {  // scratch + stream of one lm (and of a talker built on it)
    cudaStream_t stream;
    Scratch s;
    void *block;  // one allocation for all of the scratch
    int grid;
    int *h_err;   // pinned [2]
    unsigned *epoch;  // the launch epoch of this scratch's tagged words (Job::epoch)
    unsigned own_epoch = 0;
};

struct qtts_lm {
    qtts_device *dev;
    qtts_stack *stack;
    qtts_heads *heads;
    int max_pos;
    int len;
    void *k, *v;           // KV cache, float32 or (kv16) half floats
    int kv16;
    float *rope_cos, *rope_sin;
    Runner run;
    float *d_x;            // [RMAX][H] input rows
    float *h_x;            // pinned [RMAX][H]
    float *h_out;          // pinned [max rows + H]
    int max_head_rows;
    // failure-path test knobs (qtts_lm_set_wait_test): 0 = normal
    long long test_wait_cycles;
    int test_bar_extra;
};

struct qtts_talker {
    qtts_lm *talker, *pred;
    qtts_talker_config cfg;
    float *codec_emb, *pred_emb, *trailing, *tts_pad;
    int trailing_rows, trailing_cap;
    int done;  // eos chosen for the next frame
    unsigned char *seen;
    FrameState *fs, *h_fs;
    const uint8_t **d_pheads;
    int *d_hist;  // codes of qtts_talker_run: room for one frame per talker position
    size_t hist_cap;
    int step;     // FrameState.step as of the last call (frames since start)
    int started;
    SampleParams samp0, samp;  // code 0 / the predictor's codes (on = 0: greedy)
    uint64_t seed;
};

// ------------------------------------------------------------------ kernels

// f32 / bf16 rows or ggml Q8_0 blocks -> device layout (F32 rows or
// row-packed Q8_0), one thread per 32-element block; out row = r*mul + off
__global__ void pack_kernel(const void *src, int src_dtype, int rows, int k, uint8_t *dst, int dst_dtype,
                            int mul, int off) {
    const int nb = k / 32;
    long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<long long>(rows) * nb) return;
    const int r = static_cast<int>(t / nb), b = static_cast<int>(t % nb);
    const int orow = r * mul + off;
    float x[32];
    bool have_q = false;
    int8_t qv[32];
    __half dh = __float2half_rn(0.f);
    if (src_dtype == QTTS_DTYPE_F32) {
        const float *s = static_cast<const float *>(src) + static_cast<size_t>(r) * k + b * 32;
        for (int j = 0; j < 32; ++j) x[j] = s[j];
    } else if (src_dtype == QTTS_DTYPE_BF16) {
        const __nv_bfloat16 *s = static_cast<const __nv_bfloat16 *>(src) + static_cast<size_t>(r) * k + b * 32;
        for (int j = 0; j < 32; ++j) x[j] = __bfloat162float(s[j]);
    } else {
        const uint8_t *s = static_cast<const uint8_t *>(src) + (static_cast<size_t>(r) * nb + b) * 34;
        uint16_t hb = static_cast<uint16_t>(s[0] | (s[1] << 8));
        dh = __ushort_as_half(hb);
        for (int j = 0; j < 32; ++j) qv[j] = static_cast<int8_t>(s[2 + j]);
        have_q = true;
        float d = __half2float(dh);
        for (int j = 0; j < 32; ++j) x[j] = static_cast<float>(qv[j]) * d;
    }
    if (dst_dtype == QTTS_DTYPE_F32) {
        float *o = reinterpret_cast<float *>(dst + static_cast<size_t>(orow) * k * 4) + b * 32;
        for (int j = 0; j < 32; ++j) o[j] = x[j];
        return;
    }
    if (!have_q) {
        // ggml quantize_row_q8_0_ref: d = amax/127, id = 1/d, q = roundf(x*id)
        float amax = 0.f;
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
        float d = __fdiv_rn(amax, 127.0f);
        float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
        dh = __float2half_rn(d);
        for (int j = 0; j < 32; ++j) qv[j] = static_cast<int8_t>(roundf(__fmul_rn(x[j], id)));
    }
    uint8_t *row = dst + static_cast<size_t>(orow) * (k + k / 16);
    for (int j = 0; j < 32; ++j) row[b * 32 + j] = static_cast<uint8_t>(qv[j]);
    reinterpret_cast<__half *>(row + k)[b] = dh;
}

// The batch-1 kernel's layouts by kv head (its per-head phases):
// QKV rows [HKV][q(2h), q(2h+1), k(h), v(h)][H] from the [q | k | v] rows,
// one thread per 16-byte piece of a row.
__global__ void qkv_by_head_kernel(const uint8_t *src, int wdt, uint8_t *dst) {
    const int rb = row_bytes(wdt, H), pieces = rb / 16;
    const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= static_cast<long long>(QKV_ROWS) * pieces) return;
    const int row = static_cast<int>(t / pieces), pc = static_cast<int>(t % pieces);
    const int h = row / QKV_HEAD, part = (row % QKV_HEAD) / HD, i = row % HD;
    const int srow = part < 2 ? (2 * h + part) * HD + i : (part == 2 ? QDIM : QDIM + KVDIM) + h * HD + i;
    reinterpret_cast<uint4 *>(dst + static_cast<size_t>(row) * rb)[pc] =
        reinterpret_cast<const uint4 *>(src + static_cast<size_t>(srow) * rb)[pc];
}

// the O projection (row-packed [H][QDIM]) by kv head: row h*H + n = columns
// [h*KO, (h+1)*KO) of row n, with the scales of those 8 blocks (Q8_0) after
// them.  One thread per (row, block).
__global__ void oproj_by_head_kernel(const uint8_t *src, int wdt, uint8_t *dst) {
    constexpr int NB = KO / 32;  // blocks of a kv head's columns
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= HKV * H * NB) return;
    const int b = t % NB, row = t / NB;  // row of the regrouped matrix
    const int h = row / H, n = row % H;
    const int sb = h * NB + b;           // block in the source row
    if (wdt == WDT_Q8) {
        const uint8_t *srow = src + static_cast<size_t>(n) * row_bytes(WDT_Q8, QDIM);
        uint8_t *drow = dst + static_cast<size_t>(row) * row_bytes(WDT_Q8, KO);
        for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<uint32_t *>(drow + b * 32 + i) = *reinterpret_cast<const uint32_t *>(srow + sb * 32 + i);
        reinterpret_cast<uint16_t *>(drow + KO)[b] = reinterpret_cast<const uint16_t *>(srow + QDIM)[sb];
    } else {
        const float *srow = reinterpret_cast<const float *>(src + static_cast<size_t>(n) * QDIM * 4);
        float *drow = reinterpret_cast<float *>(dst + static_cast<size_t>(row) * KO * 4);
        for (int i = 0; i < 32; ++i) drow[b * 32 + i] = srow[sb * 32 + i];
    }
}

// f32 -> ggml blocks (34 bytes), the same rule
__global__ void quantize_ggml_kernel(const float *src, long long nb, uint8_t *dst) {
    long long b = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= nb) return;
    const float *x = src + b * 32;
    float amax = 0.f;
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
    float d = __fdiv_rn(amax, 127.0f);
    float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    uint8_t *o = dst + b * 34;
    // the fp16 scale as one 16-bit store (offset 34*b is even): storing its
    // two bytes separately wrote 0 for the low byte with this toolchain
    *reinterpret_cast<__half *>(o) = __float2half_rn(d);
    for (int j = 0; j < 32; ++j) o[2 + j] = static_cast<uint8_t>(static_cast<int8_t>(roundf(__fmul_rn(x[j], id))));
}

// ChooseCode0 over the talker logits after the prefill (empty history:
// eos forbidden, no penalty): one CTA
__global__ void choose0_kernel(const float *logits, int vocab, int eos, FrameState *fs) {
    __shared__ unsigned long long best[32];
    unsigned long long b = 0ull;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
        float w = logits[i];
        if (i >= vocab - 1024 && i != eos) w = -INFINITY;
        if (i == eos) w = -INFINITY;  // fewer than 2 frames
        unsigned long long k = argkey(w, i);
        b = k > b ? k : b;
    }
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long t = __shfl_xor_sync(0xffffffffu, b, o);
        b = t > b ? t : b;
    }
    if ((threadIdx.x & 31) == 0) best[threadIdx.x >> 5] = b;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long m = 0ull;
        for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) m = best[w] > m ? best[w] : m;
        int c = key_index(m);
        fs->next_code0 = c;
        fs->done = c == eos ? 1 : 0;
        fs->hist_len = 0;
        fs->step = 0;
    }
}

// ChooseCode0 after the prefill with a draw (sampling mode): the values of
// choose0_kernel, then the draw (0, 0) of the stream; NCT threads
__global__ void __launch_bounds__(NCT) choose0_sample_kernel(const float *logits, int vocab, int eos, FrameState *fs,
                                                             SampleParams p, float u) {
    __shared__ SampleScratch ss;
    const int c = sample_draw<NCT>(
        [&](int i) {
            const float w = logits[i];
            return (i >= vocab - 1024 && i != eos) || i == eos ? -INFINITY : w;  // eos: fewer than 2 frames
        },
        vocab, p, u, &ss, static_cast<int>(threadIdx.x));
    if (threadIdx.x == 0) {
        fs->next_code0 = c;
        fs->done = c == eos ? 1 : 0;
        fs->hist_len = 0;
        fs->step = 0;
    }
}

// TInferSampler.Next on values already in device memory: NCT threads
__global__ void __launch_bounds__(NCT) sample_kernel(const float *work, int n, SampleParams p, float u, int *code) {
    __shared__ SampleScratch ss;
    const int c = sample_draw<NCT>([&](int i) { return work[i]; }, n, p, u, &ss, static_cast<int>(threadIdx.x));
    if (threadIdx.x == 0) *code = c;
}

// ------------------------------------------------------------------ helpers

static bool dims_ok(const qtts_stack_config *c) {
    return c->hidden == H && c->heads == HQ && c->kv_heads == HKV && c->head_dim == HD &&
           c->intermediate == INTER && c->layers > 0;
}

static size_t src_bytes(int dtype, int rows, int k) {
    if (dtype == QTTS_DTYPE_F32) return static_cast<size_t>(rows) * k * 4;
    if (dtype == QTTS_DTYPE_BF16) return static_cast<size_t>(rows) * k * 2;
    return static_cast<size_t>(rows) * (k / 32) * 34;
}

static int ensure_staging(qtts_device *dev, size_t bytes) {
    if (dev->staging_bytes >= bytes) return QTTS_OK;
    if (dev->staging) CK(cudaFree(dev->staging));
    dev->staging = nullptr;
    dev->staging_bytes = 0;
    CK(cudaMalloc(&dev->staging, bytes));
    dev->staging_bytes = bytes;
    return QTTS_OK;
}

// upload one [rows][k] source matrix into dst (device layout), rows at r*mul+off
static int upload_matrix(qtts_device *dev, const void *src, int src_dtype, int rows, int k, uint8_t *dst,
                         int dst_dtype, int mul, int off) {
    if (!src) return set_err(QTTS_E_ARG, "missing weight matrix");
    if (src_dtype == QTTS_DTYPE_Q8_0 && dst_dtype != QTTS_DTYPE_Q8_0)
        return set_err(QTTS_E_ARG, "Q8_0 sources need Q8_0 weights");
    size_t nb = src_bytes(src_dtype, rows, k);
    int rc = ensure_staging(dev, nb);
    if (rc) return rc;
    CK(cudaMemcpyAsync(dev->staging, src, nb, cudaMemcpyHostToDevice, dev->load));
    long long n = static_cast<long long>(rows) * (k / 32);
    int threads = 256;
    unsigned blocks = static_cast<unsigned>((n + threads - 1) / threads);
    pack_kernel<<<blocks, threads, 0, dev->load>>>(dev->staging, src_dtype, rows, k, dst, dst_dtype, mul, off);
    CK(cudaGetLastError());
    CK(cudaStreamSynchronize(dev->load));
    return QTTS_OK;
}

static int upload_floats(qtts_device *dev, const float *src, size_t n, float **out, std::vector<void *> &allocs) {
    if (!src) return set_err(QTTS_E_ARG, "missing norm weights");
    CK(cudaMalloc(reinterpret_cast<void **>(out), n * 4));
    allocs.push_back(*out);
    CK(cudaMemcpy(*out, src, n * 4, cudaMemcpyHostToDevice));
    return QTTS_OK;
}

// RoPE tables as transformers computes them in float32: inv_freq_i =
// 1/theta^(2i/d), angle = pos * inv_freq_i (one float32 product), cos/sin of
// that angle
static void rope_tables(int max_pos, float theta, std::vector<float> &cs, std::vector<float> &sn) {
    const int half = HD / 2;
    cs.resize(static_cast<size_t>(max_pos) * half);
    sn.resize(static_cast<size_t>(max_pos) * half);
    for (int i = 0; i < half; ++i) {
        float e = static_cast<float>(2 * i) / static_cast<float>(HD);
        float inv = 1.0f / powf(theta, e);
        for (int p = 0; p < max_pos; ++p) {
            float a = static_cast<float>(p) * inv;
            cs[static_cast<size_t>(p) * half + i] = cosf(a);
            sn[static_cast<size_t>(p) * half + i] = sinf(a);
        }
    }
}

static uint32_t crc32c(uint32_t crc, const void *data, size_t n) {
    static uint32_t table[256];
    static bool init = false;
    if (!init) {
        for (uint32_t i = 0; i < 256; i++) {
            uint32_t c = i;
            for (int k = 0; k < 8; k++) c = c & 1 ? (c >> 1) ^ 0x82F63B78u : c >> 1;
            table[i] = c;
        }
        init = true;
    }
    const uint8_t *p = static_cast<const uint8_t *>(data);
    crc = ~crc;
    for (size_t i = 0; i < n; i++) crc = table[(crc ^ p[i]) & 0xff] ^ (crc >> 8);
    return ~crc;
}

// ------------------------------------------------------------------ tcgen05 GEMM (host)

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int encode_init() {
    if (!g_encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (!fn || q != cudaDriverEntryPointSuccess) return set_err(QTTS_E_CUDA, "cuTensorMapEncodeTiled not found");
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    return QTTS_OK;
}

static int tensor_map_f16(CUtensorMap *map, const __half *base, int k, int rows_cap, int box_rows) {
    int rc0 = encode_init();
    if (rc0) return rc0;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows_cap)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(G_BK), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_err(QTTS_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return QTTS_OK;
}

template <int WDT, int BN>
static int gemm_attr() {
    // the CTAs of one SM share its 228 KB (1 KB of it reserved per CTA)
    static_assert(g_ctas_per_sm(WDT, BN) * (sizeof(GemmSmem<WDT, BN>) + 1024 + 1024) <= 228 * 1024,
                  "GEMM CTAs per SM exceed the shared memory");
    CK(cudaFuncSetAttribute(gemm_kernel<WDT, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            static_cast<int>(sizeof(GemmSmem<WDT, BN>) + 1024)));
    CK(cudaFuncSetAttribute(gemm_kernel<WDT, BN>, cudaFuncAttributePreferredSharedMemoryCarveout,
                            cudaSharedmemCarveoutMaxShared));
    return QTTS_OK;
}

// kernel attributes and the tensor-map encoder, once per device (before
// any stream capture, where they could not be set)
static int gemm_init(qtts_device *dev) {
    static std::mutex mu;
    static bool done[256] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (dev->ordinal >= 0 && dev->ordinal < 256 && done[dev->ordinal]) return QTTS_OK;
    int rc;
    if ((rc = gemm_attr<WDT_Q8, 64>()) || (rc = gemm_attr<WDT_Q8, 128>()) || (rc = gemm_attr<WDT_Q8, 256>()) ||
        (rc = gemm_attr<WDT_F32, 64>()) || (rc = gemm_attr<WDT_F32, 128>()) || (rc = gemm_attr<WDT_F32, 256>()))
        return rc;
    CK(cudaFuncSetAttribute(attn_prefill_tc_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            static_cast<int>(sizeof(TaSmem) + 1024)));
    CK(cudaFuncSetAttribute(attn_prefill_tc_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            static_cast<int>(sizeof(TaSmem) + 1024)));
    CK(cudaFuncSetAttribute(attn_decode_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            static_cast<int>(sizeof(DecodeSmem<float>))));
    CK(cudaFuncSetAttribute(attn_decode_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            static_cast<int>(sizeof(DecodeSmem<__nv_bfloat16>))));
    if ((rc = encode_init())) return rc;
    if (dev->ordinal >= 0 && dev->ordinal < 256) done[dev->ordinal] = true;
    return QTTS_OK;
}

template <int WDT, int BN>
static int gemm_launch_t(const GemmArgs &a, const __half *x, int rows_cap, dim3 grid, cudaStream_t st) {
    const size_t smem = sizeof(GemmSmem<WDT, BN>) + 1024;
    CUtensorMap map;
    int rc = tensor_map_f16(&map, x, a.K, rows_cap, BN);
    if (rc) return rc;
    if (grid.z > 1)
        CK(launch_pdl_cluster(gemm_kernel<WDT, BN>, grid, dim3(g_threads(WDT)), smem, st, grid.z, a, map));
    else
        CK(launch_pdl(gemm_kernel<WDT, BN>, grid, dim3(g_threads(WDT)), smem, st, a, map));
    return QTTS_OK;
}

// y[t][n] (+)= x[t][:] . w[n][:] for t < T (w tile-packed; x: fp16 [rows_cap][K] on the
// device, rows_cap >= T).  With `add`, the products are added to y (residual);
// otherwise y is overwritten.
// tokens per tile: float32 weights stop at 128 (two CTAs per SM, one's
// epilogue under the other's main loop)
static int gemm_bn(int T, int wdt) { return T <= 64 ? 64 : (T <= 128 || wdt == WDT_F32 ? 128 : 256); }

// the K split of a GEMM: CTAs up to about one per SM, at most 8 per tile
// (a portable cluster; clusters of 16 measured slower: 9.38 vs 7.79 ms per
// B=64 frame)
static int gemm_split(int n_rows, int k, int T, int wdt) {
    const int cap = 8;
    const int bn = gemm_bn(T, wdt);
    const int tiles = ((n_rows + G_BM - 1) / G_BM) * ((T + bn - 1) / bn);
    const int kb = k / G_BK;
    int split = 1;
    while (split * 2 <= cap && split * 2 <= kb && kb % (split * 2) == 0 && tiles * split * 2 <= 160) split *= 2;
    return split;
}

// y[t][n] (+)= ...  A K split sums its partials in a fixed order inside a
// cluster (no atomics, no cleared output).  With swiglu16 (gate/up pairs in
// consecutive rows), fp16(silu(gate) * up) goes to swiglu16[t][n / 2] (row
// stride ld) instead of y.
// the QKV projection's fused epilogue (GemmArgs::q32 and what follows it)
struct QkvEpi {
    float *q32;
    const float *q_norm, *k_norm, *rope_cos, *rope_sin;
    float eps;
    const int *tok_seq, *tok_pos;
    void *kv_base;
    const int *kv_pages;
    int kv_mpps, kv_layers, kv_layer, kv_bf16;
    __half *kv16;  // the fp16 mirror of the pages, or NULL
};

static int gemm(const uint8_t *w, int wdt, int n_rows, int k, const __half *x, int T, int rows_cap, float *y, int ld,
                bool add, int *err, cudaStream_t st, __half *swiglu16 = nullptr, const QkvEpi *qe = nullptr) {
    if (k % G_BK != 0) return set_err(QTTS_E_ARG, "gemm: K %d is not a multiple of %d", k, G_BK);
    const int bn = gemm_bn(T, wdt);
    const int split = gemm_split(n_rows, k, T, wdt);
    GemmArgs a;
    a.w = w;
    a.n_rows = n_rows;
    a.K = k;
    a.T = T;
    a.out = y;
    a.ld = ld;
    a.atomic = add ? 1 : 0;
    a.ksplit = split;
    a.err = err;
    a.swiglu16 = swiglu16;
    a.ld16 = swiglu16 ? ld : 0;
    a.q32 = nullptr;
    a.q_norm = a.k_norm = a.rope_cos = a.rope_sin = nullptr;
    a.eps = 0.f;
    a.tok_seq = a.tok_pos = nullptr;
    a.kv_base = nullptr;
    a.kv_pages = nullptr;
    a.kv_mpps = a.kv_layers = a.kv_layer = a.kv_bf16 = 0;
    a.kv16 = nullptr;
    if (qe) {
        if (n_rows != QKV_ROWS) return set_err(QTTS_E_ARG, "gemm: the QKV epilogue needs the %d QKV rows", QKV_ROWS);
        a.q32 = qe->q32;
        a.q_norm = qe->q_norm;
        a.k_norm = qe->k_norm;
        a.rope_cos = qe->rope_cos;
        a.rope_sin = qe->rope_sin;
        a.eps = qe->eps;
        a.tok_seq = qe->tok_seq;
        a.tok_pos = qe->tok_pos;
        a.kv_base = qe->kv_base;
        a.kv_pages = qe->kv_pages;
        a.kv_mpps = qe->kv_mpps;
        a.kv_layers = qe->kv_layers;
        a.kv_layer = qe->kv_layer;
        a.kv_bf16 = qe->kv_bf16;
        a.kv16 = qe->kv16;
    }
    dim3 grid((n_rows + G_BM - 1) / G_BM, (T + bn - 1) / bn, split);
    if (wdt == WDT_Q8) {
        if (bn == 64) return gemm_launch_t<WDT_Q8, 64>(a, x, rows_cap, grid, st);
        if (bn == 128) return gemm_launch_t<WDT_Q8, 128>(a, x, rows_cap, grid, st);
        return gemm_launch_t<WDT_Q8, 256>(a, x, rows_cap, grid, st);
    }
    if (bn == 64) return gemm_launch_t<WDT_F32, 64>(a, x, rows_cap, grid, st);
    if (bn == 128) return gemm_launch_t<WDT_F32, 128>(a, x, rows_cap, grid, st);
    return gemm_launch_t<WDT_F32, 256>(a, x, rows_cap, grid, st);
}

// the tile-packed copy of a row-packed matrix (freed by the caller)
static int tile_pack(const uint8_t *src, int wdt, int n_rows, int k, uint8_t **out) {
    *out = nullptr;
    const size_t bytes = static_cast<size_t>((n_rows + G_BM - 1) / G_BM) * (k / G_BK) * g_chunk_bytes(wdt);
    if (cudaMalloc(out, bytes) != cudaSuccess) return set_err(QTTS_E_OOM, "gemm tiles: out of device memory");
    const long long n = static_cast<long long>((n_rows + G_BM - 1) / G_BM * G_BM) * (k / G_BK) * 8;
    gemm_tile_pack_kernel<<<static_cast<unsigned>((n + 255) / 256), 256>>>(src, wdt, n_rows, k, *out);
    if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(*out);
        *out = nullptr;
        return set_err(QTTS_E_CUDA, "gemm tiles: packing failed");
    }
    return QTTS_OK;
}

// ------------------------------------------------------------------ device

extern "C" int qtts_device_open(int ordinal, qtts_device **out) {
    if (!out) return set_err(QTTS_E_ARG, "qtts_device_open: out is NULL");
    *out = nullptr;
    int n = 0;
    CK(cudaGetDeviceCount(&n));
    if (ordinal < 0 || ordinal >= n) return set_err(QTTS_E_ARG, "qtts_device_open: no CUDA device %d (%d)", ordinal, n);
    CK(cudaSetDevice(ordinal));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, ordinal));
    if (prop.major < 10) return set_err(QTTS_E_ARG, "qtts_device_open: %s is sm_%d%d, sm_100a needed", prop.name, prop.major, prop.minor);
    if (!prop.cooperativeLaunch) return set_err(QTTS_E_ARG, "qtts_device_open: no cooperative launch");
    if (prop.multiProcessorCount * XS_MAX < H || prop.multiProcessorCount < 128)
        return set_err(QTTS_E_ARG, "qtts_device_open: %d SMs is too few", prop.multiProcessorCount);
    size_t smem = sizeof(Smem) + 128;
    CK(cudaFuncSetAttribute(decode_kernel<WDT_F32, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    CK(cudaFuncSetAttribute(decode_kernel<WDT_Q8, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    CK(cudaFuncSetAttribute(decode_kernel<WDT_F32, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    CK(cudaFuncSetAttribute(decode_kernel<WDT_Q8, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    int occ = 0, occ16 = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_kernel<WDT_Q8, 0>, NTHREADS, smem));
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ16, decode_kernel<WDT_Q8, 1>, NTHREADS, smem));
    occ = occ < occ16 ? occ : occ16;
    if (occ < 1) return set_err(QTTS_E_CUDA, "qtts_device_open: the decode kernel does not fit on an SM");
    qtts_device *d = new qtts_device();
    d->ordinal = ordinal;
    d->sms = prop.multiProcessorCount;
    d->smem = smem;
    d->staging = nullptr;
    d->staging_bytes = 0;
    d->bytes = 0;
    snprintf(d->name, sizeof(d->name), "%s", prop.name);
    cudaError_t e = cudaStreamCreateWithFlags(&d->load, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete d;
        return set_err(QTTS_E_CUDA, "cudaStreamCreate: %s", cudaGetErrorString(e));
    }
    *out = d;
    return QTTS_OK;
}

extern "C" int qtts_device_name(qtts_device *dev, char *buf, int len) {
    if (!dev || !buf || len <= 0) return set_err(QTTS_E_ARG, "qtts_device_name: bad argument");
    snprintf(buf, len, "%s", dev->name);
    return QTTS_OK;
}

extern "C" int qtts_device_bytes(qtts_device *dev, int64_t *bytes) {
    if (!dev || !bytes) return set_err(QTTS_E_ARG, "qtts_device_bytes: bad argument");
    *bytes = dev->bytes;
    return QTTS_OK;
}

extern "C" int qtts_device_close(qtts_device *dev) {
    if (!dev) return QTTS_OK;
    cudaSetDevice(dev->ordinal);
    if (dev->staging) cudaFree(dev->staging);
    if (dev->draw_in) cudaFree(dev->draw_in);
    cudaStreamDestroy(dev->load);
    delete dev;
    return QTTS_OK;
}

// ------------------------------------------------------------------ stack

static void stack_free(qtts_stack *s) {
    for (void *p : s->allocs) cudaFree(p);
    delete s;
}

// The matrices of layer l into its device buffers (wqkv [QKV_ROWS], wo,
// wgu [gate/up interleaved], wd, in the stack's format), and its four norms
// (float32 host pointers: input, post, q, k).
struct LayerFill {
    virtual int matrices(int l, uint8_t *wqkv, uint8_t *wo, uint8_t *wgu, uint8_t *wd) = 0;
    virtual void norms(int l, const float *n[4]) = 0;
};

// One Qwen3 stack on the device from `fill`: allocations, the batch-1
// per-head layouts, the norms and the layer table
static int stack_build(qtts_device *dev, const qtts_stack_config *c, LayerFill &fill, const float *final_norm,
                       qtts_stack **out) {
    CK(cudaSetDevice(dev->ordinal));
    qtts_stack *s = new qtts_stack();
    s->dev = dev;
    s->cfg = *c;
    s->d_layers = nullptr;
    const int wdt = c->dtype == QTTS_DTYPE_F32 ? WDT_F32 : WDT_Q8;
    std::vector<DLayer> hl(c->layers);
    int rc = QTTS_OK;
    auto alloc = [&](size_t bytes) -> uint8_t * {
        void *p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
        s->allocs.push_back(p);
        return static_cast<uint8_t *>(p);
    };
    int64_t mat_bytes = 0;
    for (int l = 0; l < c->layers && rc == QTTS_OK; ++l) {
        DLayer &d = hl[l];
        size_t bqkv = static_cast<size_t>(QKV_ROWS) * row_bytes(wdt, H);
        size_t bo = static_cast<size_t>(H) * row_bytes(wdt, QDIM);
        size_t bgu = static_cast<size_t>(GU_ROWS) * row_bytes(wdt, H);
        size_t bd = static_cast<size_t>(H) * row_bytes(wdt, INTER);
        size_t boh = static_cast<size_t>(HKV) * H * row_bytes(wdt, KO);
        uint8_t *wqkv = alloc(bqkv), *wo = alloc(bo), *wgu = alloc(bgu), *wd = alloc(bd);
        uint8_t *wqkvh = alloc(bqkv), *woh = alloc(boh);
        if (!wqkv || !wo || !wgu || !wd || !wqkvh || !woh) {
            rc = set_err(QTTS_E_OOM, "qtts_stack_create: out of device memory at layer %d", l);
            break;
        }
        mat_bytes += bqkv + bo + bgu + bd;
        if ((rc = fill.matrices(l, wqkv, wo, wgu, wd))) break;
        {
            const long long nq = static_cast<long long>(QKV_ROWS) * (row_bytes(wdt, H) / 16);
            qkv_by_head_kernel<<<static_cast<unsigned>((nq + 255) / 256), 256, 0, dev->load>>>(wqkv, wdt, wqkvh);
            oproj_by_head_kernel<<<(HKV * H * (KO / 32) + 255) / 256, 256, 0, dev->load>>>(wo, wdt, woh);
            if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(dev->load) != cudaSuccess) {
                rc = set_err(QTTS_E_CUDA, "qtts_stack_create: per-head layouts failed at layer %d", l);
                break;
            }
        }
        d.wqkv = wqkv;
        d.wo = wo;
        d.wqkvh = wqkvh;
        d.woh = woh;
        d.wgu = wgu;
        d.wd = wd;
        const float *n[4];
        fill.norms(l, n);
        float *p;
        if ((rc = upload_floats(dev, n[0], H, &p, s->allocs))) break;
        d.in_norm = p;
        if ((rc = upload_floats(dev, n[1], H, &p, s->allocs))) break;
        d.post_norm = p;
        if ((rc = upload_floats(dev, n[2], HD, &p, s->allocs))) break;
        d.q_norm = p;
        if ((rc = upload_floats(dev, n[3], HD, &p, s->allocs))) break;
        d.k_norm = p;
    }
    if (rc == QTTS_OK) rc = upload_floats(dev, final_norm, H, &s->d_final_norm, s->allocs);
    if (rc == QTTS_OK) {
        uint8_t *dl = alloc(sizeof(DLayer) * c->layers);
        if (!dl)
            rc = set_err(QTTS_E_OOM, "qtts_stack_create: out of device memory");
        else if (cudaMemcpy(dl, hl.data(), sizeof(DLayer) * c->layers, cudaMemcpyHostToDevice) != cudaSuccess)
            rc = set_err(QTTS_E_CUDA, "qtts_stack_create: layer table upload failed");
        s->d_layers = reinterpret_cast<DLayer *>(dl);
        s->hlayers = hl;
    }
    if (rc != QTTS_OK) {
        stack_free(s);
        return rc;
    }
    // StackBytes (lm.pas:181-197): matrices + (2 hidden + 2 head_dim) norms
    // per layer + the final norm
    s->bytes = mat_bytes + (static_cast<int64_t>(2 * H + 2 * HD) * 4) * c->layers + H * 4;
    // stacks that fit comfortably in L2 keep their lines (evict_last)
    s->keep_l2 = mat_bytes <= (96ll << 20) ? 1 : 0;
    dev->bytes += s->bytes;
    *out = s;
    return QTTS_OK;
}

extern "C" int qtts_stack_create(qtts_device *dev, const qtts_stack_config *c, const qtts_layer_src *layers,
                                 const float *final_norm, qtts_stack **out) {
    if (!dev || !c || !layers || !final_norm || !out) return set_err(QTTS_E_ARG, "qtts_stack_create: NULL argument");
    *out = nullptr;
    if (!dims_ok(c))
        return set_err(QTTS_E_ARG, "qtts_stack_create: unsupported dimensions (hidden %d, heads %d/%d, head_dim %d, intermediate %d, layers %d)",
                       c->hidden, c->heads, c->kv_heads, c->head_dim, c->intermediate, c->layers);
    if (c->dtype != QTTS_DTYPE_F32 && c->dtype != QTTS_DTYPE_Q8_0)
        return set_err(QTTS_E_ARG, "qtts_stack_create: weights must be F32 or Q8_0");
    for (int l = 0; l < c->layers; ++l) {
        const int sd = layers[l].dtype;
        if (sd != QTTS_DTYPE_F32 && sd != QTTS_DTYPE_BF16 && sd != QTTS_DTYPE_Q8_0)
            return set_err(QTTS_E_ARG, "qtts_stack_create: layer %d has dtype %d", l, sd);
    }
    // host rows (F32, BF16 or ggml Q8_0 blocks), converted on the device
    struct HostFill : LayerFill {
        qtts_device *dev;
        const qtts_layer_src *layers;
        int dt;
        int matrices(int l, uint8_t *wqkv, uint8_t *wo, uint8_t *wgu, uint8_t *wd) override {
            const qtts_layer_src &a = layers[l];
            const int sd = a.dtype;
            int rc;
            if ((rc = upload_matrix(dev, a.q_proj, sd, QDIM, H, wqkv, dt, 1, 0))) return rc;
            if ((rc = upload_matrix(dev, a.k_proj, sd, KVDIM, H, wqkv, dt, 1, QDIM))) return rc;
            if ((rc = upload_matrix(dev, a.v_proj, sd, KVDIM, H, wqkv, dt, 1, QDIM + KVDIM))) return rc;
            if ((rc = upload_matrix(dev, a.o_proj, sd, H, QDIM, wo, dt, 1, 0))) return rc;
            if ((rc = upload_matrix(dev, a.gate_proj, sd, INTER, H, wgu, dt, 2, 0))) return rc;
            if ((rc = upload_matrix(dev, a.up_proj, sd, INTER, H, wgu, dt, 2, 1))) return rc;
            return upload_matrix(dev, a.down_proj, sd, H, INTER, wd, dt, 1, 0);
        }
        void norms(int l, const float *n[4]) override {
            n[0] = layers[l].input_norm;
            n[1] = layers[l].post_norm;
            n[2] = layers[l].q_norm;
            n[3] = layers[l].k_norm;
        }
    } fill;
    fill.dev = dev;
    fill.layers = layers;
    fill.dt = c->dtype;
    return stack_build(dev, c, fill, final_norm, out);
}

extern "C" int qtts_stack_bytes(const qtts_stack *s, int64_t *bytes) {
    if (!s || !bytes) return set_err(QTTS_E_ARG, "qtts_stack_bytes: bad argument");
    *bytes = s->bytes;
    return QTTS_OK;
}

extern "C" int qtts_stack_destroy(qtts_stack *s) {
    if (!s) return QTTS_OK;
    cudaSetDevice(s->dev->ordinal);
    s->dev->bytes -= s->bytes;
    stack_free(s);
    return QTTS_OK;
}

// ------------------------------------------------------------------ heads

extern "C" int qtts_heads_create(qtts_device *dev, const char *name, int hidden, int dtype, qtts_heads **out) {
    if (!dev || !out) return set_err(QTTS_E_ARG, "qtts_heads_create: NULL argument");
    *out = nullptr;
    if (dtype != QTTS_DTYPE_F32 && dtype != QTTS_DTYPE_Q8_0)
        return set_err(QTTS_E_ARG, "qtts_heads_create: %s weights not supported", dtype == QTTS_DTYPE_BF16 ? "BF16" : "unknown");
    if (hidden <= 0 || (hidden & 31) != 0)
        return set_err(QTTS_E_ARG, "qtts_heads_create: invalid width %d for %s", hidden, name ? name : "");
    if (hidden != H) return set_err(QTTS_E_ARG, "qtts_heads_create: width %d, the stacks have %d", hidden, H);
    qtts_heads *h = new qtts_heads();
    h->dev = dev;
    h->name = name ? name : "";
    h->hidden = hidden;
    h->dtype = dtype;
    h->bytes = 0;
    *out = h;
    return QTTS_OK;
}

extern "C" int qtts_heads_add(qtts_heads *h, const void *src, int src_dtype, int rows, int *index) {
    if (!h || !src) return set_err(QTTS_E_ARG, "qtts_heads_add: NULL argument");
    if (rows <= 0) return set_err(QTTS_E_ARG, "qtts_heads_add: %d rows", rows);
    if (src_dtype != QTTS_DTYPE_F32 && src_dtype != QTTS_DTYPE_BF16 && src_dtype != QTTS_DTYPE_Q8_0)
        return set_err(QTTS_E_ARG, "qtts_heads_add: source dtype %d", src_dtype);
    CK(cudaSetDevice(h->dev->ordinal));
    const int wdt = h->dtype == QTTS_DTYPE_F32 ? WDT_F32 : WDT_Q8;
    size_t bytes = static_cast<size_t>(rows) * row_bytes(wdt, h->hidden);
    uint8_t *d = nullptr;
    CK(cudaMalloc(&d, bytes));
    int rc = upload_matrix(h->dev, src, src_dtype, rows, h->hidden, d, h->dtype, 1, 0);
    if (rc) {
        cudaFree(d);
        return rc;
    }
    h->mats.push_back({d, rows, nullptr});
    // TQwenLmHeads.Bytes counts the stored bytes (ggml blocks: 34 per 32)
    h->bytes += static_cast<int64_t>(rows) * (h->dtype == QTTS_DTYPE_F32 ? h->hidden * 4 : h->hidden / 32 * 34);
    if (index) *index = static_cast<int>(h->mats.size()) - 1;
    return QTTS_OK;
}

extern "C" int qtts_heads_digest(qtts_heads *h, uint32_t *crc) {
    if (!h || !crc) return set_err(QTTS_E_ARG, "qtts_heads_digest: NULL argument");
    CK(cudaSetDevice(h->dev->ordinal));
    uint32_t c = 0;
    const int k = h->hidden;
    for (const HeadMat &m : h->mats) {
        if (h->dtype == QTTS_DTYPE_F32) {
            std::vector<uint8_t> buf(static_cast<size_t>(m.rows) * k * 4);
            CK(cudaMemcpy(buf.data(), m.d, buf.size(), cudaMemcpyDeviceToHost));
            c = crc32c(c, buf.data(), buf.size());
        } else {
            // row-packed -> ggml blocks, in order
            size_t rb = static_cast<size_t>(k) + k / 16;
            std::vector<uint8_t> buf(static_cast<size_t>(m.rows) * rb);
            CK(cudaMemcpy(buf.data(), m.d, buf.size(), cudaMemcpyDeviceToHost));
            std::vector<uint8_t> g(static_cast<size_t>(m.rows) * (k / 32) * 34);
            for (int r = 0; r < m.rows; ++r)
                for (int b = 0; b < k / 32; ++b) {
                    const uint8_t *row = buf.data() + r * rb;
                    uint8_t *o = g.data() + (static_cast<size_t>(r) * (k / 32) + b) * 34;
                    o[0] = row[k + 2 * b];
                    o[1] = row[k + 2 * b + 1];
                    memcpy(o + 2, row + b * 32, 32);
                }
            c = crc32c(c, g.data(), g.size());
        }
    }
    *crc = c;
    return QTTS_OK;
}

extern "C" int qtts_heads_count(qtts_heads *h, int *count) {
    if (!h || !count) return set_err(QTTS_E_ARG, "qtts_heads_count: NULL argument");
    *count = static_cast<int>(h->mats.size());
    return QTTS_OK;
}

extern "C" int qtts_heads_rows(qtts_heads *h, int index, int *rows) {
    if (!h || !rows) return set_err(QTTS_E_ARG, "qtts_heads_rows: NULL argument");
    if (index < 0 || index >= static_cast<int>(h->mats.size()))
        return set_err(QTTS_E_ARG, "qtts_heads_rows: no head %d", index);
    *rows = h->mats[index].rows;
    return QTTS_OK;
}

extern "C" int qtts_heads_bytes(qtts_heads *h, int64_t *bytes) {
    if (!h || !bytes) return set_err(QTTS_E_ARG, "qtts_heads_bytes: NULL argument");
    *bytes = h->bytes;
    return QTTS_OK;
}

static int heads_tiles(qtts_heads *h) {
    const int wdt = h->dtype == QTTS_DTYPE_F32 ? WDT_F32 : WDT_Q8;
    for (HeadMat &m : h->mats) {
        if (m.t) continue;
        int rc = tile_pack(m.d, wdt, m.rows, h->hidden, &m.t);
        if (rc) return rc;
    }
    return QTTS_OK;
}

static int stack_tiles(qtts_stack *s) {
    if (!s->tlayers.empty()) return QTTS_OK;
    const int wdt = s->cfg.dtype == QTTS_DTYPE_F32 ? WDT_F32 : WDT_Q8;
    std::vector<DLayer> tl(s->hlayers);
    for (DLayer &d : tl) {
        struct M {
            const uint8_t **p;
            int rows, k;
        } ms[] = {{&d.wqkv, QKV_ROWS, H}, {&d.wo, H, QDIM}, {&d.wgu, GU_ROWS, H}, {&d.wd, H, INTER}};
        for (const M &m : ms) {
            uint8_t *t = nullptr;
            int rc = tile_pack(*m.p, wdt, m.rows, m.k, &t);
            if (rc) return rc;
            s->allocs.push_back(t);
            *m.p = t;
        }
    }
    s->tlayers = tl;
    return QTTS_OK;
}

extern "C" int qtts_heads_linear(qtts_heads *h, int index, const float *x, int rows, float *y) {
    if (!h || !x || !y) return set_err(QTTS_E_ARG, "qtts_heads_linear: NULL argument");
    if (index < 0 || index >= static_cast<int>(h->mats.size()))
        return set_err(QTTS_E_ARG, "qtts_heads_linear: no head %d in %s", index, h->name.c_str());
    if (rows <= 0) return QTTS_OK;
    CK(cudaSetDevice(h->dev->ordinal));
    int rc = gemm_init(h->dev);
    if (rc == QTTS_OK) rc = heads_tiles(h);
    if (rc) return rc;
    const HeadMat &m = h->mats[index];
    const int k = h->hidden;
    cudaStream_t st = h->dev->load;
    if (static_cast<size_t>(rows) > h->lrows) {
        if (h->lx) CK(cudaFree(h->lx));
        if (h->lh) CK(cudaFree(h->lh));
        h->lx = nullptr;
        h->lh = nullptr;
        h->lrows = 0;
        CK(cudaMalloc(&h->lx, static_cast<size_t>(rows) * k * 4));
        CK(cudaMalloc(&h->lh, static_cast<size_t>(rows) * k * 2));
        h->lrows = rows;
    }
    const size_t ny = static_cast<size_t>(rows) * m.rows;
    if (ny > h->lycap) {
        if (h->ly) CK(cudaFree(h->ly));
        h->ly = nullptr;
        h->lycap = 0;
        CK(cudaMalloc(&h->ly, ny * 4));
        h->lycap = ny;
    }
    if (!h->lerr) CK(cudaMalloc(&h->lerr, 16));
    CK(cudaMemsetAsync(h->lerr, 0, 16, st));
    const long long n = static_cast<long long>(rows) * k;
    CK(cudaMemcpyAsync(h->lx, x, n * 4, cudaMemcpyHostToDevice, st));
    to_half_kernel<<<static_cast<unsigned>((n / 4 + 255) / 256), 256, 0, st>>>(h->lx, h->lh, n);
    CK(cudaGetLastError());
    const int wdt = h->dtype == QTTS_DTYPE_F32 ? WDT_F32 : WDT_Q8;
    rc = gemm(m.t, wdt, m.rows, k, h->lh, rows, static_cast<int>(h->lrows), h->ly, m.rows, false, h->lerr, st);
    if (rc) return rc;
    int err = 0;
    CK(cudaMemcpyAsync(&err, h->lerr, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(y, h->ly, ny * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (err) return set_err(QTTS_E_TIMEOUT, "qtts_heads_linear: a device wait gave up");
    return QTTS_OK;
}

extern "C" int qtts_heads_destroy(qtts_heads *h) {
    if (!h) return QTTS_OK;
    cudaSetDevice(h->dev->ordinal);
    for (HeadMat &m : h->mats) {
        cudaFree(m.d);
        if (m.t) cudaFree(m.t);
    }
    if (h->lx) cudaFree(h->lx);
    if (h->ly) cudaFree(h->ly);
    if (h->lh) cudaFree(h->lh);
    if (h->lerr) cudaFree(h->lerr);
    delete h;
    return QTTS_OK;
}

// ------------------------------------------------------------------ runner

static int runner_init(Runner &r, qtts_device *dev, int max_head_rows) {
    r.grid = dev->sms;
    const int maxS = r.grid / HKV;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        size_t o = off;
        off += (bytes + 255) & ~static_cast<size_t>(255);
        return o;
    };
    size_t ox = take(RMAX * H * 4), ox8 = take(RMAX * H * 8), oqkv = take(RMAX * QKV_ROWS * 8),
           oact = take(RMAX * INTER * 4),
           opart = take(static_cast<size_t>(HKV) * maxS * RMAX * 2 * PSTRIDE * 4),
           oarg = take(static_cast<size_t>(r.grid) * 8), obar = take(BAR_WORDS * 4), oerr = take(16),
           olog = take(static_cast<size_t>(max_head_rows) * 4), ohid = take(H * 4), oxt = take(H * 4);
    CK(cudaStreamCreateWithFlags(&r.stream, cudaStreamNonBlocking));
    CK(cudaMalloc(&r.block, off));
    CK(cudaMemset(r.block, 0, off));
    uint8_t *b = static_cast<uint8_t *>(r.block);
    r.s.x = reinterpret_cast<float *>(b + ox);
    r.s.x8 = reinterpret_cast<unsigned long long *>(b + ox8);
    r.s.qkv = reinterpret_cast<unsigned long long *>(b + oqkv);
    r.s.act = reinterpret_cast<float *>(b + oact);
    r.epoch = &r.own_epoch;
    r.own_epoch = 0;
    r.s.part = reinterpret_cast<float *>(b + opart);
    r.s.arg = reinterpret_cast<unsigned long long *>(b + oarg);
    r.s.bar = reinterpret_cast<unsigned *>(b + obar);
    r.s.err = reinterpret_cast<int *>(b + oerr);
    r.s.logits = reinterpret_cast<float *>(b + olog);
    r.s.hidden = reinterpret_cast<float *>(b + ohid);
    r.s.xt = reinterpret_cast<float *>(b + oxt);
    CK(cudaMallocHost(reinterpret_cast<void **>(&r.h_err), 16));
    return QTTS_OK;
}

static void runner_free(Runner &r) {
    if (r.block) cudaFree(r.block);
    if (r.h_err) cudaFreeHost(r.h_err);
    if (r.stream) cudaStreamDestroy(r.stream);
    r.block = nullptr;
    r.h_err = nullptr;
    r.stream = nullptr;
}

static int launch(qtts_device *dev, Runner &r, const Job &job_in, int wdt) {
    // a new epoch for the tags of this launch's handoffs; before an epoch
    // comes round again, the tagged words are cleared (tag 0 is never used)
    Job job = job_in;
    if (++*r.epoch >= EPOCH_LIMIT) {
        CK(cudaMemsetAsync(r.s.x8, 0, static_cast<size_t>(RMAX) * H * 8, r.stream));
        CK(cudaMemsetAsync(r.s.qkv, 0, static_cast<size_t>(RMAX) * QKV_ROWS * 8, r.stream));
        *r.epoch = 1;
    }
    job.epoch = *r.epoch;
    void *args[] = {&job};
    // the cache format of the launch: the lm's, or the talker's (whose
    // predictor holds the same, qtts_talker_create)
    const int kv16 = job.mode == 0 ? job.ctx.kv16 : job.tctx.kv16;
    const void *fn = wdt == WDT_F32 ? (kv16 ? reinterpret_cast<const void *>(decode_kernel<WDT_F32, 1>)
                                            : reinterpret_cast<const void *>(decode_kernel<WDT_F32, 0>))
                                    : (kv16 ? reinterpret_cast<const void *>(decode_kernel<WDT_Q8, 1>)
                                            : reinterpret_cast<const void *>(decode_kernel<WDT_Q8, 0>));
    CK(cudaLaunchCooperativeKernel(fn, dim3(r.grid), dim3(NTHREADS), args, dev->smem, r.stream));
    return QTTS_OK;
}

// after a launch: read the error word; on a device error, clear the
// counters so that the next launch starts clean
static int runner_check(Runner &r) {
    CK(cudaMemcpyAsync(r.h_err, r.s.err, 8, cudaMemcpyDeviceToHost, r.stream));
    CK(cudaStreamSynchronize(r.stream));
    if (r.h_err[0] != 0) {
        int code = r.h_err[0], where = r.h_err[1];
        CK(cudaMemsetAsync(r.s.err, 0, 16, r.stream));
        CK(cudaMemsetAsync(r.s.bar, 0, BAR_WORDS * 4, r.stream));
        CK(cudaStreamSynchronize(r.stream));
        return set_err(code == ERR_CAPACITY ? QTTS_E_CAPACITY : QTTS_E_TIMEOUT,
                       "device wait gave up (code %d at %d): the kernel returned early", code, where);
    }
    return QTTS_OK;
}

static DStack dstack(const qtts_stack *s) {
    DStack d;
    d.layer = s->d_layers;
    d.layers = s->cfg.layers;
    d.eps = s->cfg.rms_eps;
    d.final_norm = s->d_final_norm;
    d.keep_l2 = s->keep_l2;
    return d;
}

// ------------------------------------------------------------------ lm

static void lm_free(qtts_lm *m) {
    if (m->k) cudaFree(m->k);
    if (m->v) cudaFree(m->v);
    if (m->rope_cos) cudaFree(m->rope_cos);
    if (m->rope_sin) cudaFree(m->rope_sin);
    if (m->d_x) cudaFree(m->d_x);
    if (m->h_x) cudaFreeHost(m->h_x);
    if (m->h_out) cudaFreeHost(m->h_out);
    runner_free(m->run);
    delete m;
}

static void *noalloc_lookup(int ordinal);

static int lm_create(qtts_stack *stack, qtts_heads *heads, int max_pos, int kv_dtype, qtts_lm **out) {
    if (!stack || !heads || !out) return set_err(QTTS_E_ARG, "qtts_lm_create: NULL argument");
    if (kv_dtype != QTTS_DTYPE_F32 && kv_dtype != QTTS_DTYPE_F16)
        return set_err(QTTS_E_ARG, "qtts_lm_create: KV cache in F32 or F16");
    *out = nullptr;
    if (heads->hidden != stack->cfg.hidden)
        return set_err(QTTS_E_ARG, "qtts_lm_create: %s has a width of %d, its heads %d", heads->name.c_str(),
                       stack->cfg.hidden, heads->hidden);
    if (heads->dtype != stack->cfg.dtype)
        return set_err(QTTS_E_ARG, "qtts_lm_create: heads and stack have different weight formats");
    if (max_pos <= 0 || max_pos > (1 << 20)) return set_err(QTTS_E_ARG, "qtts_lm_create: max_pos %d", max_pos);
    qtts_device *dev = stack->dev;
    CK(cudaSetDevice(dev->ordinal));
    qtts_lm *m = new qtts_lm();
    m->dev = dev;
    m->stack = nullptr;
    m->heads = heads;
    m->max_pos = max_pos;
    m->len = 0;
    m->kv16 = kv_dtype == QTTS_DTYPE_F16 ? 1 : 0;
    m->max_head_rows = 4096;
    for (const HeadMat &hm : heads->mats) m->max_head_rows = hm.rows > m->max_head_rows ? hm.rows : m->max_head_rows;
    int rc = QTTS_OK;
    size_t kvn = static_cast<size_t>(stack->cfg.layers) * HKV * max_pos * HD;
    std::vector<float> cs, sn;
    rope_tables(max_pos, stack->cfg.rope_theta, cs, sn);
    const size_t kvb = m->kv16 ? 2 : 4;
    if (cudaMalloc(&m->k, kvn * kvb) != cudaSuccess || cudaMalloc(&m->v, kvn * kvb) != cudaSuccess ||
        cudaMalloc(&m->rope_cos, cs.size() * 4) != cudaSuccess || cudaMalloc(&m->rope_sin, sn.size() * 4) != cudaSuccess ||
        cudaMalloc(&m->d_x, RMAX * H * 4) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void **>(&m->h_x), RMAX * H * 4) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void **>(&m->h_out), (m->max_head_rows + H) * 4) != cudaSuccess) {
        rc = set_err(QTTS_E_OOM, "qtts_lm_create: out of memory (KV cache of %d positions)", max_pos);
    }
    if (rc == QTTS_OK && (cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
                          cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess))
        rc = set_err(QTTS_E_CUDA, "qtts_lm_create: RoPE upload failed");
    if (rc == QTTS_OK) rc = runner_init(m->run, dev, m->max_head_rows);
    if (rc != QTTS_OK) {
        lm_free(m);
        return rc;
    }
    m->stack = stack;  // owned from here on
    // the device address of qtts_lm_forward_noalloc's static scratch, taken
    // here (set-up, this device current) so that those calls load nothing;
    // a failure is not this call's: the first such call retries and reports
    (void)noalloc_lookup(dev->ordinal);
    *out = m;
    return QTTS_OK;
}

extern "C" int qtts_lm_create(qtts_stack *stack, qtts_heads *heads, int max_pos, qtts_lm **out) {
    return lm_create(stack, heads, max_pos, QTTS_DTYPE_F32, out);
}

extern "C" int qtts_lm_create_kv(qtts_stack *stack, qtts_heads *heads, int max_pos, int kv_dtype, qtts_lm **out) {
    return lm_create(stack, heads, max_pos, kv_dtype, out);
}

extern "C" int qtts_lm_set_launch_epoch(qtts_lm *m, uint32_t epoch) {
    if (!m || !m->run.epoch || epoch >= EPOCH_LIMIT)
        return set_err(QTTS_E_ARG, "qtts_lm_set_launch_epoch: bad argument (epoch below %u)", EPOCH_LIMIT);
    *m->run.epoch = epoch;
    return QTTS_OK;
}

extern "C" int qtts_lm_set_wait_test(qtts_lm *m, int extra_arrivals, int64_t wait_cycles) {
    if (!m || extra_arrivals < 0 || extra_arrivals > 1 || wait_cycles < 0)
        return set_err(QTTS_E_ARG, "qtts_lm_set_wait_test: bad argument");
    m->test_bar_extra = extra_arrivals;
    m->test_wait_cycles = wait_cycles;
    return QTTS_OK;
}

extern "C" int qtts_lm_reset(qtts_lm *m) {
    if (!m) return set_err(QTTS_E_ARG, "qtts_lm_reset: NULL lm");
    m->len = 0;
    return QTTS_OK;
}

extern "C" int qtts_lm_length(qtts_lm *m, int *length) {
    if (!m || !length) return set_err(QTTS_E_ARG, "qtts_lm_length: NULL argument");
    *length = m->len;
    return QTTS_OK;
}

static Job base_job(qtts_lm *m) {
    Job j;
    memset(&j, 0, sizeof(j));
    j.s = m->run.s;
    j.rope_cos = m->rope_cos;
    j.rope_sin = m->rope_sin;
    j.rope_pos = m->max_pos;
    j.wait_cycles = m->test_wait_cycles > 0 ? m->test_wait_cycles : WAIT_CYCLES;
    j.bar_extra = m->test_bar_extra;
    return j;
}

// x: host rows, or device rows when x_dev (the prompt built on the device)
static int lm_forward(qtts_lm *m, const float *x, bool x_dev, int rows, int head, float *logits, float *hidden) {
    if (!m) return set_err(QTTS_E_ARG, "qtts_lm_forward: NULL lm");
    if (rows <= 0) return QTTS_OK;
    if (!x) return set_err(QTTS_E_ARG, "qtts_lm_forward: x is NULL");
    if (logits && (head < 0 || head >= static_cast<int>(m->heads->mats.size())))
        return set_err(QTTS_E_ARG, "qtts_lm_forward: no head %d in %s", head, m->heads->name.c_str());
    if (m->len + rows > m->max_pos)
        return set_err(QTTS_E_CAPACITY, "qtts_lm_forward: %d + %d positions, the cache holds %d", m->len, rows,
                       m->max_pos);
    CK(cudaSetDevice(m->dev->ordinal));
    const int wdt = m->stack->cfg.dtype == QTTS_DTYPE_F32 ? WDT_F32 : WDT_Q8;
    Job j = base_job(m);
    j.mode = 0;
    j.st = dstack(m->stack);
    j.ctx.k = m->k;
    j.ctx.v = m->v;
    j.ctx.kv16 = m->kv16;
    j.ctx.max_pos = m->max_pos;
    j.xin = m->d_x;
    // RMAX rows per launch; the head and the normed state come from the last
    for (int r0 = 0; r0 < rows; r0 += RMAX) {
        int n = rows - r0 < RMAX ? rows - r0 : RMAX;
        bool last = r0 + n == rows;
        if (x_dev) {
            CK(cudaMemcpyAsync(m->d_x, x + static_cast<size_t>(r0) * H, static_cast<size_t>(n) * H * 4,
                               cudaMemcpyDeviceToDevice, m->run.stream));
        } else {
            memcpy(m->h_x, x + static_cast<size_t>(r0) * H, static_cast<size_t>(n) * H * 4);
            CK(cudaMemcpyAsync(m->d_x, m->h_x, static_cast<size_t>(n) * H * 4, cudaMemcpyHostToDevice, m->run.stream));
        }
        j.rows = n;
        j.L0 = m->len;
        j.head_w = (last && logits) ? m->heads->mats[head].d : nullptr;
        j.head_rows = (last && logits) ? m->heads->mats[head].rows : 0;
        int rc = launch(m->dev, m->run, j, wdt);
        if (rc) return rc;
        // positions are appended whatever happens next (the cache is written)
        rc = runner_check(m->run);
        if (rc) return rc;
        m->len += n;
    }
    int hr = logits ? m->heads->mats[head].rows : 0;
    if (logits) CK(cudaMemcpyAsync(m->h_out, m->run.s.logits, hr * 4, cudaMemcpyDeviceToHost, m->run.stream));
    if (hidden) CK(cudaMemcpyAsync(m->h_out + m->max_head_rows, m->run.s.hidden, H * 4, cudaMemcpyDeviceToHost, m->run.stream));
    CK(cudaStreamSynchronize(m->run.stream));
    if (logits) memcpy(logits, m->h_out, hr * 4);
    if (hidden) memcpy(hidden, m->h_out + m->max_head_rows, H * 4);
    return QTTS_OK;
}

extern "C" int qtts_lm_forward(qtts_lm *m, const float *x, int rows, int head, float *logits, float *hidden) {
    return lm_forward(m, x, false, rows, head, logits, hidden);
}

extern "C" int qtts_lm_destroy(qtts_lm *m) {
    if (!m) return QTTS_OK;
    cudaSetDevice(m->dev->ordinal);
    qtts_stack *s = m->stack;
    lm_free(m);
    qtts_stack_destroy(s);
    return QTTS_OK;
}

// ------------------------------------------------------------------ talker

static void talker_free(qtts_talker *t) {
    if (t->codec_emb) cudaFree(t->codec_emb);
    if (t->pred_emb) cudaFree(t->pred_emb);
    if (t->trailing) cudaFree(t->trailing);
    if (t->tts_pad) cudaFree(t->tts_pad);
    if (t->seen) cudaFree(t->seen);
    if (t->fs) cudaFree(t->fs);
    if (t->h_fs) cudaFreeHost(t->h_fs);
    if (t->d_pheads) cudaFree(t->d_pheads);
    if (t->d_hist) cudaFree(t->d_hist);
    delete t;
}

extern "C" int qtts_talker_create(qtts_lm *talker, qtts_lm *pred, const qtts_talker_config *c, const float *codec_emb,
                                  const float *pred_emb, qtts_talker **out) {
    if (!talker || !pred || !c || !codec_emb || !pred_emb || !out)
        return set_err(QTTS_E_ARG, "qtts_talker_create: NULL argument");
    *out = nullptr;
    if (talker->dev != pred->dev) return set_err(QTTS_E_ARG, "qtts_talker_create: the stacks are on two devices");
    if (talker->stack->cfg.dtype != pred->stack->cfg.dtype)
        return set_err(QTTS_E_ARG, "qtts_talker_create: talker and predictor have different weight formats");
    if (talker->stack->cfg.rope_theta != pred->stack->cfg.rope_theta)
        return set_err(QTTS_E_ARG, "qtts_talker_create: talker and predictor have different RoPE bases");
    if (talker->kv16 != pred->kv16)
        return set_err(QTTS_E_ARG, "qtts_talker_create: talker and predictor caches of different formats");
    if (c->groups < 2 || c->groups > MAX_GROUPS) return set_err(QTTS_E_ARG, "qtts_talker_create: %d code groups", c->groups);
    if (c->vocab <= 1024 || c->pred_vocab <= 0 || c->codec_eos < 0 || c->codec_eos >= c->vocab)
        return set_err(QTTS_E_ARG, "qtts_talker_create: unexpected vocabularies (%d, %d, eos %d)", c->vocab, c->pred_vocab,
                       c->codec_eos);
    if (talker->heads->mats.size() < 1 || talker->heads->mats[0].rows != c->vocab)
        return set_err(QTTS_E_ARG, "qtts_talker_create: the talker head must have %d rows", c->vocab);
    if (static_cast<int>(pred->heads->mats.size()) < c->groups - 1)
        return set_err(QTTS_E_ARG, "qtts_talker_create: the predictor needs %d heads", c->groups - 1);
    for (int g = 0; g < c->groups - 1; ++g)
        if (pred->heads->mats[g].rows != c->pred_vocab)
            return set_err(QTTS_E_ARG, "qtts_talker_create: predictor head %d has %d rows", g, pred->heads->mats[g].rows);
    if (pred->max_pos < c->groups || talker->max_pos < c->groups)
        return set_err(QTTS_E_ARG, "qtts_talker_create: the caches must hold at least %d positions", c->groups);
    CK(cudaSetDevice(talker->dev->ordinal));
    qtts_talker *t = new qtts_talker();
    t->talker = talker;
    t->pred = pred;
    t->cfg = *c;
    size_t ne = static_cast<size_t>(c->vocab) * H, np = static_cast<size_t>(c->groups - 1) * c->pred_vocab * H;
    int rc = QTTS_OK;
    if (cudaMalloc(&t->codec_emb, ne * 4) != cudaSuccess || cudaMalloc(&t->pred_emb, np * 4) != cudaSuccess ||
        cudaMalloc(&t->tts_pad, H * 4) != cudaSuccess || cudaMalloc(&t->seen, c->vocab) != cudaSuccess ||
        cudaMalloc(&t->fs, sizeof(FrameState)) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void **>(&t->h_fs), sizeof(FrameState)) != cudaSuccess ||
        cudaMalloc(&t->d_pheads, sizeof(uint8_t *) * (c->groups - 1)) != cudaSuccess ||
        cudaMalloc(&t->d_hist, static_cast<size_t>(talker->max_pos) * c->groups * 4) != cudaSuccess)
        rc = set_err(QTTS_E_OOM, "qtts_talker_create: out of device memory");
    t->hist_cap = static_cast<size_t>(talker->max_pos) * c->groups;
    if (rc == QTTS_OK) {
        std::vector<const uint8_t *> ph(c->groups - 1);
        for (int g = 0; g < c->groups - 1; ++g) ph[g] = pred->heads->mats[g].d;
        if (cudaMemcpy(t->codec_emb, codec_emb, ne * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(t->pred_emb, pred_emb, np * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(t->d_pheads, ph.data(), sizeof(uint8_t *) * ph.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemset(t->fs, 0, sizeof(FrameState)) != cudaSuccess || cudaMemset(t->seen, 0, c->vocab) != cudaSuccess)
            rc = set_err(QTTS_E_CUDA, "qtts_talker_create: upload failed");
    }
    if (rc != QTTS_OK) {
        talker_free(t);
        return rc;
    }
    *out = t;
    return QTTS_OK;
}

// rows_dev: prefill, trailing and tts_pad are device rows (the prompt built
// on the device, on the talker's stream), else host rows
static int talker_start(qtts_talker *t, bool rows_dev, const float *prefill, int rows, const float *trailing,
                        int trailing_rows, const float *tts_pad, float *logits, float *hidden) {
    const cudaMemcpyKind kind = rows_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    qtts_lm *tl = t->talker;
    CK(cudaSetDevice(tl->dev->ordinal));
    cudaStream_t st = tl->run.stream;
    if (trailing_rows > t->trailing_cap) {
        if (t->trailing) CK(cudaFree(t->trailing));
        t->trailing = nullptr;
        CK(cudaMalloc(&t->trailing, static_cast<size_t>(trailing_rows) * H * 4));
        t->trailing_cap = trailing_rows;
    }
    if (trailing_rows > 0)
        CK(cudaMemcpyAsync(t->trailing, trailing, static_cast<size_t>(trailing_rows) * H * 4, kind, st));
    t->trailing_rows = trailing_rows;
    CK(cudaMemcpyAsync(t->tts_pad, tts_pad, H * 4, kind, st));
    CK(cudaMemsetAsync(t->seen, 0, t->cfg.vocab, st));
    t->started = 0;
    // TQwenTalker.Start: fTalker.Reset; fTalker.Forward(prefill, rows, 0, ...)
    qtts_lm_reset(tl);
    // the head always runs: the first ChooseCode0 reads its logits
    std::vector<float> tmp(logits ? 0 : t->cfg.vocab);
    int rc = lm_forward(tl, prefill, rows_dev, rows, 0, logits ? logits : tmp.data(), hidden);
    if (rc) return rc;
    // the first ChooseCode0 (empty history): the argmax or the draw (0, 0);
    // then the frame state
    if (t->samp0.on)
        choose0_sample_kernel<<<1, NCT, 0, st>>>(tl->run.s.logits, t->cfg.vocab, t->cfg.codec_eos, t->fs, t->samp0,
                                                 sample_uniform(t->seed, 0, 0));
    else
        choose0_kernel<<<1, 1024, 0, st>>>(tl->run.s.logits, t->cfg.vocab, t->cfg.codec_eos, t->fs);
    CK(cudaGetLastError());
    FrameState h;
    CK(cudaMemcpyAsync(&h, t->fs, sizeof(h), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    h.tlen = tl->len;
    CK(cudaMemcpyAsync(t->fs, &h, sizeof(h), cudaMemcpyHostToDevice, st));
    CK(cudaStreamSynchronize(st));
    t->done = h.done;
    t->step = h.step;
    t->started = 1;
    return QTTS_OK;
}

extern "C" int qtts_talker_start(qtts_talker *t, const float *prefill, int rows, const float *trailing, int trailing_rows,
                                 const float *tts_pad, float *logits, float *hidden) {
    if (!t || !prefill || !tts_pad || rows <= 0 || trailing_rows < 0 || (trailing_rows > 0 && !trailing))
        return set_err(QTTS_E_ARG, "qtts_talker_start: bad argument");
    return talker_start(t, false, prefill, rows, trailing, trailing_rows, tts_pad, logits, hidden);
}

static Job frame_job(qtts_talker *t) {
    qtts_lm *tl = t->talker, *pl = t->pred;
    Job j = base_job(tl);
    j.mode = 1;
    j.tst = dstack(tl->stack);
    j.pst = dstack(pl->stack);
    j.tctx.k = tl->k;
    j.tctx.v = tl->v;
    j.tctx.kv16 = tl->kv16;
    j.tctx.max_pos = tl->max_pos;
    j.pctx.k = pl->k;
    j.pctx.v = pl->v;
    j.pctx.kv16 = pl->kv16;
    j.pctx.max_pos = pl->max_pos;
    j.theads = tl->heads->mats[0].d;
    j.tvocab = t->cfg.vocab;
    j.pheads = t->d_pheads;
    j.pvocab = t->cfg.pred_vocab;
    j.groups = t->cfg.groups;
    j.codec_emb = t->codec_emb;
    j.pred_emb = t->pred_emb;
    j.trailing = t->trailing;
    j.trailing_rows = t->trailing_rows;
    j.tts_pad = t->tts_pad;
    j.eos = t->cfg.codec_eos;
    j.penalty = t->cfg.repetition_penalty;
    j.seen = t->seen;
    j.samp0 = t->samp0;
    j.samp = t->samp;
    j.seed = t->seed;
    j.fs = t->fs;
    j.codes_hist = nullptr;
    j.codes_cap = 0;
    j.trace = nullptr;
    j.trace_cap = 0;
    j.trace_n = nullptr;
    return j;
}

static int next_frame(qtts_talker *t, int32_t *codes, int *more, uint64_t *stamps, int cap, int *n);

extern "C" int qtts_talker_next_frame(qtts_talker *t, int32_t *codes, int *more) {
    return next_frame(t, codes, more, nullptr, 0, nullptr);
}

extern "C" int qtts_talker_trace_frame(qtts_talker *t, int32_t *codes, int *more, uint64_t *stamps, int cap, int *n) {
    if (!stamps || cap <= 0 || !n) return set_err(QTTS_E_ARG, "qtts_talker_trace_frame: bad trace buffer");
    *n = 0;
    return next_frame(t, codes, more, stamps, cap, n);
}

static int next_frame(qtts_talker *t, int32_t *codes, int *more, uint64_t *stamps, int cap, int *n) {
    if (!t || !codes || !more) return set_err(QTTS_E_ARG, "qtts_talker_next_frame: NULL argument");
    if (!t->started) return set_err(QTTS_E_STATE, "qtts_talker_next_frame: call qtts_talker_start first");
    qtts_lm *tl = t->talker, *pl = t->pred;
    if (t->done) {  // ChooseCode0 gave eos: NextFrame returns false
        *more = 0;
        return QTTS_OK;
    }
    if (tl->len + 1 > tl->max_pos)
        return set_err(QTTS_E_CAPACITY, "qtts_talker_next_frame: the talker cache is full (%d positions)", tl->max_pos);
    CK(cudaSetDevice(tl->dev->ordinal));
    const int wdt = tl->stack->cfg.dtype == QTTS_DTYPE_F32 ? WDT_F32 : WDT_Q8;
    Job j = frame_job(t);
    unsigned long long *d_trace = nullptr;
    if (stamps) {
        CK(cudaMalloc(&d_trace, (static_cast<size_t>(cap) + 1) * 8));
        j.trace = d_trace;
        j.trace_cap = cap;
        j.trace_n = reinterpret_cast<int *>(d_trace + cap);
        CK(cudaMemset(j.trace_n, 0, 4));
    }
    int rc = launch(tl->dev, tl->run, j, wdt);
    if (rc) {
        if (d_trace) cudaFree(d_trace);
        return rc;
    }
    CK(cudaMemcpyAsync(t->h_fs, t->fs, sizeof(FrameState), cudaMemcpyDeviceToHost, tl->run.stream));
    rc = runner_check(tl->run);
    if (d_trace) {
        int cnt = 0;
        cudaMemcpy(&cnt, j.trace_n, 4, cudaMemcpyDeviceToHost);
        cnt = cnt < cap ? cnt : cap;
        cudaMemcpy(stamps, d_trace, static_cast<size_t>(cnt) * 8, cudaMemcpyDeviceToHost);
        *n = cnt;
        cudaFree(d_trace);
    }
    if (rc) return rc;
    const FrameState &f = *t->h_fs;
    if (f.tlen == tl->len) {  // eos was chosen before this frame: nothing ran
        t->done = 1;
        *more = 0;
        return QTTS_OK;
    }
    for (int g = 0; g < t->cfg.groups; ++g) codes[g] = f.codes[g];
    t->done = f.done;
    t->step = f.step;
    tl->len = f.tlen;
    pl->len = t->cfg.groups;
    *more = 1;
    return QTTS_OK;
}

extern "C" int qtts_talker_run(qtts_talker *t, int frames, int32_t *codes, int *produced) {
    if (!t || !produced || frames < 0 || (frames > 0 && !codes)) return set_err(QTTS_E_ARG, "qtts_talker_run: bad argument");
    if (!t->started) return set_err(QTTS_E_STATE, "qtts_talker_run: call qtts_talker_start first");
    *produced = 0;
    qtts_lm *tl = t->talker, *pl = t->pred;
    if (t->done || frames == 0) return QTTS_OK;
    if (tl->len + frames > tl->max_pos)
        return set_err(QTTS_E_CAPACITY, "qtts_talker_run: %d + %d positions, the talker cache holds %d", tl->len, frames,
                       tl->max_pos);
    CK(cudaSetDevice(tl->dev->ordinal));
    const int wdt = tl->stack->cfg.dtype == QTTS_DTYPE_F32 ? WDT_F32 : WDT_Q8;
    // each frame takes one talker position, so the history buffer made at
    // create (max_pos frames) holds the run: nothing is allocated or read
    // back before the launches
    if (static_cast<size_t>(frames) * t->cfg.groups > t->hist_cap)
        return set_err(QTTS_E_CAPACITY, "qtts_talker_run: %d frames, room for %zu", frames, t->hist_cap / t->cfg.groups);
    const int step0 = t->step;
    Job j = frame_job(t);
    // frame f is written at row (step0 + f) - step0: shift the base pointer
    j.codes_hist = t->d_hist - static_cast<ptrdiff_t>(step0) * t->cfg.groups;
    j.codes_cap = step0 + frames;
    for (int f = 0; f < frames; ++f) {
        int rc = launch(tl->dev, tl->run, j, wdt);
        if (rc) return rc;
    }
    CK(cudaMemcpyAsync(t->h_fs, t->fs, sizeof(FrameState), cudaMemcpyDeviceToHost, tl->run.stream));
    int rc = runner_check(tl->run);
    if (rc) return rc;
    const FrameState &f = *t->h_fs;
    int n = f.step - step0;
    if (n > 0) CK(cudaMemcpy(codes, t->d_hist, static_cast<size_t>(n) * t->cfg.groups * 4, cudaMemcpyDeviceToHost));
    *produced = n;
    t->done = f.done;
    t->step = f.step;
    tl->len = f.tlen;
    if (n > 0) pl->len = t->cfg.groups;
    return QTTS_OK;
}

extern "C" int qtts_talker_stream(qtts_talker *t, void **stream) {
    if (!t || !stream) return set_err(QTTS_E_ARG, "qtts_talker_stream: NULL argument");
    *stream = static_cast<void *>(t->talker->run.stream);
    return QTTS_OK;
}

extern "C" int qtts_talker_probe(qtts_talker *t, float *logits, float *hidden) {
    if (!t) return set_err(QTTS_E_ARG, "qtts_talker_probe: NULL talker");
    if (!t->started) return set_err(QTTS_E_STATE, "qtts_talker_probe: call qtts_talker_start first");
    qtts_lm *tl = t->talker;
    CK(cudaSetDevice(tl->dev->ordinal));
    if (logits) CK(cudaMemcpy(logits, tl->run.s.logits, static_cast<size_t>(t->cfg.vocab) * 4, cudaMemcpyDeviceToHost));
    if (hidden) CK(cudaMemcpy(hidden, tl->run.s.hidden, H * 4, cudaMemcpyDeviceToHost));
    return QTTS_OK;
}

extern "C" int qtts_talker_step(qtts_talker *t, int *step) {
    if (!t || !step) return set_err(QTTS_E_ARG, "qtts_talker_step: NULL argument");
    if (!t->started) {
        *step = 0;
        return QTTS_OK;
    }
    CK(cudaSetDevice(t->talker->dev->ordinal));
    FrameState h;
    CK(cudaMemcpy(&h, t->fs, sizeof(h), cudaMemcpyDeviceToHost));
    *step = h.step;
    return QTTS_OK;
}

extern "C" int qtts_talker_destroy(qtts_talker *t) {
    if (!t) return QTTS_OK;
    cudaSetDevice(t->talker->dev->ordinal);
    talker_free(t);
    return QTTS_OK;
}

static int sampling_params(const char *who, int on, float temperature, int top_k, float top_p, SampleParams *out) {
    out->on = on ? 1 : 0;
    out->temperature = temperature;
    out->top_k = top_k;
    out->top_p = top_p;
    if (!on) return QTTS_OK;
    if (!(temperature > 0.0f) || top_k < 1 || top_k > SAMPLE_MAX_K || !(top_p > 0.0f) || !(top_p <= 1.0f))
        return set_err(QTTS_E_ARG, "%s: temperature %g, top_k %d, top_p %g (need > 0, 1..%d, (0, 1])", who,
                       static_cast<double>(temperature), top_k, static_cast<double>(top_p), SAMPLE_MAX_K);
    return QTTS_OK;
}

extern "C" int qtts_talker_set_sampling(qtts_talker *t, const qtts_sampling *s) {
    if (!t || !s) return set_err(QTTS_E_ARG, "qtts_talker_set_sampling: NULL argument");
    SampleParams a, b;
    int rc = sampling_params("qtts_talker_set_sampling", s->do_sample, s->temperature, s->top_k, s->top_p, &a);
    if (rc) return rc;
    rc = sampling_params("qtts_talker_set_sampling (predictor)", s->sub_do_sample, s->sub_temperature,
                         s->sub_top_k, s->sub_top_p, &b);
    if (rc) return rc;
    if (t->cfg.vocab > SAMPLE_MAX_V || t->cfg.pred_vocab > SAMPLE_MAX_V)
        return set_err(QTTS_E_ARG, "qtts_talker_set_sampling: vocabularies of %d / %d, at most %d", t->cfg.vocab,
                       t->cfg.pred_vocab, SAMPLE_MAX_V);
    t->samp0 = a;
    t->samp = b;
    t->seed = s->seed;
    return QTTS_OK;
}

extern "C" int qtts_sample(qtts_device *dev, const float *work, int n, float temperature, int top_k, float top_p,
                           uint64_t seed, int step, int group, int32_t *code) {
    if (!dev || !work || !code) return set_err(QTTS_E_ARG, "qtts_sample: NULL argument");
    if (n <= 0 || n > SAMPLE_MAX_V) return set_err(QTTS_E_ARG, "qtts_sample: %d values (1..%d)", n, SAMPLE_MAX_V);
    SampleParams p;
    int rc = sampling_params("qtts_sample", 1, temperature, top_k, top_p, &p);
    if (rc) return rc;
    CK(cudaSetDevice(dev->ordinal));
    // the values and the code in one buffer of the device object, made on
    // the first draw (draws on one device are serialised by the caller)
    if (!dev->draw_in && cudaMalloc(&dev->draw_in, (SAMPLE_MAX_V + 1) * 4) != cudaSuccess) {
        dev->draw_in = nullptr;
        return set_err(QTTS_E_OOM, "qtts_sample: out of device memory");
    }
    float *d = dev->draw_in;
    int *dc = reinterpret_cast<int *>(d + SAMPLE_MAX_V);
    cudaError_t e = cudaMemcpy(d, work, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        sample_kernel<<<1, NCT>>>(d, n, p, sample_uniform(seed, step, group), dc);
        e = cudaGetLastError();
    }
    int c = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&c, dc, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return set_err(QTTS_E_CUDA, "qtts_sample: %s", cudaGetErrorString(e));
    *code = c;
    return QTTS_OK;
}

// ------------------------------------------------------------------ utilities

// ------------------------------------------------------------------ text projection
//
// TQwenTalker.TextProject (talker.pas:390-421): Qwen3TTSTalkerResizeMLP,
// y = fc2(silu(fc1(text_embedding[id]))), float32 with biases, the rows of
// the prompt and of the trailing text (talker.pas:532-574).  The embedding
// table stays on the device in its source format (BF16 as in the
// checkpoint, or float32); fc1 / fc2 in float32.

struct qtts_textproj {
    qtts_device *dev;
    int vocab, text_hidden, hidden, emb_dtype;
    void *emb;
    float *w1, *b1, *w2, *b2;
    float *e, *h, *y;  // [cap][text_hidden] x2, [cap][hidden]
    int *ids;
    int cap;
};

// e[r][k] = emb[ids[r]][k] widened to float32; ids checked on the host
__global__ void text_gather_kernel(const void *emb, int dtype, int kdim, const int *ids, int n, float *e) {
    const int r = blockIdx.x;
    if (r >= n) return;
    const size_t row = static_cast<size_t>(ids[r]) * kdim;
    for (int k = threadIdx.x; k < kdim; k += blockDim.x)
        e[static_cast<size_t>(r) * kdim + k] = dtype == QTTS_DTYPE_BF16
                                                   ? __bfloat162float(static_cast<const __nv_bfloat16 *>(emb)[row + k])
                                                   : static_cast<const float *>(emb)[row + k];
}

// y[r][o] = sum_k x[r][k] w[o][k] + b[o] (then silu as TextProject: 0 below
// -80, else v / (1 + exp(-v))): a warp per output o, its weight row in
// registers (kdim <= 32 * TP_KPL), the rows of x streamed.  With codec, row
// r then gets codec_emb[codec[r]][o] added when codec[r] >= 0 (AddRow of
// Start, talker.pas:423-429, over the projected row).
constexpr int TP_KPL = 64;
__global__ void __launch_bounds__(256) text_linear_kernel(const float *x, int n, int kdim, const float *w,
                                                         const float *b, int odim, int silu, float *y,
                                                         const int *codec = nullptr,
                                                         const float *codec_emb = nullptr) {
    const int o = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (o >= odim) return;
    float wr[TP_KPL];
#pragma unroll
    for (int j = 0; j < TP_KPL; ++j) {
        const int k = lane + 32 * j;
        wr[j] = k < kdim ? w[static_cast<size_t>(o) * kdim + k] : 0.f;
    }
    const float bo = b[o];
    for (int r = 0; r < n; ++r) {
        const float *xr = x + static_cast<size_t>(r) * kdim;
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < TP_KPL; ++j) {
            const int k = lane + 32 * j;
            if (k < kdim) acc = fmaf(wr[j], xr[k], acc);
        }
#pragma unroll
        for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
        if (lane == 0) {
            float v = acc + bo;
            if (silu) v = v < -80.f ? 0.f : v / (1.0f + expf(-v));
            if (codec && codec[r] >= 0) v += codec_emb[static_cast<size_t>(codec[r]) * odim + o];
            y[static_cast<size_t>(r) * odim + o] = v;
        }
    }
}

static void textproj_free(qtts_textproj *t) {
    for (void *p : {t->emb, static_cast<void *>(t->w1), static_cast<void *>(t->b1), static_cast<void *>(t->w2),
                    static_cast<void *>(t->b2), static_cast<void *>(t->e), static_cast<void *>(t->h),
                    static_cast<void *>(t->y), static_cast<void *>(t->ids)})
        if (p) cudaFree(p);
    delete t;
}

extern "C" int qtts_textproj_create(qtts_device *dev, int vocab, int text_hidden, int hidden, int emb_dtype,
                                    const void *emb, const float *fc1_w, const float *fc1_b, const float *fc2_w,
                                    const float *fc2_b, qtts_textproj **out) {
    if (!dev || !emb || !fc1_w || !fc1_b || !fc2_w || !fc2_b || !out)
        return set_err(QTTS_E_ARG, "qtts_textproj_create: NULL argument");
    *out = nullptr;
    if (vocab <= 0 || text_hidden <= 0 || text_hidden > 32 * TP_KPL || hidden <= 0)
        return set_err(QTTS_E_ARG, "qtts_textproj_create: vocab %d, text hidden %d (1..%d), hidden %d", vocab,
                       text_hidden, 32 * TP_KPL, hidden);
    if (emb_dtype != QTTS_DTYPE_F32 && emb_dtype != QTTS_DTYPE_BF16)
        return set_err(QTTS_E_ARG, "qtts_textproj_create: embedding dtype %d (F32 or BF16)", emb_dtype);
    CK(cudaSetDevice(dev->ordinal));
    qtts_textproj *t = new qtts_textproj();
    t->dev = dev;
    t->vocab = vocab;
    t->text_hidden = text_hidden;
    t->hidden = hidden;
    t->emb_dtype = emb_dtype;
    const size_t eb = static_cast<size_t>(vocab) * text_hidden * (emb_dtype == QTTS_DTYPE_BF16 ? 2 : 4);
    const size_t w1 = static_cast<size_t>(text_hidden) * text_hidden * 4, w2 = static_cast<size_t>(hidden) * text_hidden * 4;
    cudaError_t e = cudaMalloc(&t->emb, eb);
    if (e == cudaSuccess) e = cudaMalloc(&t->w1, w1);
    if (e == cudaSuccess) e = cudaMalloc(&t->b1, static_cast<size_t>(text_hidden) * 4);
    if (e == cudaSuccess) e = cudaMalloc(&t->w2, w2);
    if (e == cudaSuccess) e = cudaMalloc(&t->b2, static_cast<size_t>(hidden) * 4);
    if (e == cudaSuccess) e = cudaMemcpy(t->emb, emb, eb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(t->w1, fc1_w, w1, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(t->b1, fc1_b, static_cast<size_t>(text_hidden) * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(t->w2, fc2_w, w2, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(t->b2, fc2_b, static_cast<size_t>(hidden) * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        textproj_free(t);
        return set_err(e == cudaErrorMemoryAllocation ? QTTS_E_OOM : QTTS_E_CUDA, "qtts_textproj_create: %s",
                       cudaGetErrorString(e));
    }
    *out = t;
    return QTTS_OK;
}

// t->y[n][hidden] = the projections of the text tokens ids[n] (host, checked
// by the caller), each plus codec_emb[codec[r]] where codec (host, or NULL)
// gives one >= 0; ids and codec go up on `st`, which then holds the work
static int textproj_run(qtts_textproj *t, const int32_t *ids, const int32_t *codec, const float *codec_emb, int n,
                        cudaStream_t st) {
    CK(cudaSetDevice(t->dev->ordinal));
    if (n > t->cap) {
        CK(cudaStreamSynchronize(st));
        for (void *p : {static_cast<void *>(t->e), static_cast<void *>(t->h), static_cast<void *>(t->y),
                        static_cast<void *>(t->ids)})
            if (p) cudaFree(p);
        t->e = t->h = t->y = nullptr;
        t->ids = nullptr;
        t->cap = 0;
        cudaError_t e = cudaMalloc(&t->e, static_cast<size_t>(n) * t->text_hidden * 4);
        if (e == cudaSuccess) e = cudaMalloc(&t->h, static_cast<size_t>(n) * t->text_hidden * 4);
        if (e == cudaSuccess) e = cudaMalloc(&t->y, static_cast<size_t>(n) * t->hidden * 4);
        if (e == cudaSuccess) e = cudaMalloc(&t->ids, static_cast<size_t>(n) * 2 * 4);  // ids, then codec
        if (e != cudaSuccess) return set_err(QTTS_E_OOM, "qtts_text_project: %s", cudaGetErrorString(e));
        t->cap = n;
    }
    int *d_codec = t->ids + t->cap;
    CK(cudaMemcpyAsync(t->ids, ids, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, st));
    if (codec) CK(cudaMemcpyAsync(d_codec, codec, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, st));
    text_gather_kernel<<<n, 256, 0, st>>>(t->emb, t->emb_dtype, t->text_hidden, t->ids, n, t->e);
    text_linear_kernel<<<(t->text_hidden + 7) / 8, 256, 0, st>>>(t->e, n, t->text_hidden, t->w1, t->b1,
                                                                 t->text_hidden, 1, t->h);
    text_linear_kernel<<<(t->hidden + 7) / 8, 256, 0, st>>>(t->h, n, t->text_hidden, t->w2, t->b2, t->hidden, 0,
                                                            t->y, codec ? d_codec : nullptr, codec_emb);
    CK(cudaGetLastError());
    return QTTS_OK;
}

extern "C" int qtts_text_project(qtts_textproj *t, const int32_t *ids, int n, float *y) {
    if (!t || (n > 0 && (!ids || !y))) return set_err(QTTS_E_ARG, "qtts_text_project: NULL argument");
    if (n <= 0) return QTTS_OK;
    for (int r = 0; r < n; ++r)
        if (ids[r] < 0 || ids[r] >= t->vocab)
            return set_err(QTTS_E_ARG, "qtts_text_project: text token %d out of range", ids[r]);
    int rc = textproj_run(t, ids, nullptr, nullptr, n, 0);
    if (rc) return rc;
    CK(cudaMemcpy(y, t->y, static_cast<size_t>(n) * t->hidden * 4, cudaMemcpyDeviceToHost));
    return QTTS_OK;
}

// ------------------------------------------------------------------ the prompt of Start

// The rows of TQwenTalker.Start (talker.pas:528-574), each as (text token,
// codec id or -1): every row is the projection of one text token (the role,
// the text, or tts_pad / tts_bos / tts_eos, whose vectors are projections
// too, talker.pas:339-344), plus one codec embedding for the rows over the
// codec.  Listed in the order prefill rows, trailing rows, then tts_pad (the
// row after the trailing text).
struct PromptPlan {
    std::vector<int32_t> text, codec;
    int rows = 0, trailing = 0;
};

// the rows alone (host logic, no device): ids and codec counts checked
static int plan_rows(const char *fn, const qtts_prompt_tokens *tok, const int32_t *ids, int n_ids,
                     const int32_t *codec, int n_codec, int non_streaming, PromptPlan &p) {
    if (!tok || !ids || !codec) return set_err(QTTS_E_ARG, "%s: NULL argument", fn);
    // [im_start, assistant, \n] text [im_end, \n, im_start, assistant, \n]
    if (n_ids < 9) return set_err(QTTS_E_ARG, "%s: empty text (%d prompt ids, at least 9)", fn, n_ids);
    if (n_codec < 2) return set_err(QTTS_E_ARG, "%s: %d codec ids (at least pad and bos)", fn, n_codec);
    auto row = [&p](int32_t text, int32_t c) {
        p.text.push_back(text);
        p.codec.push_back(c);
    };
    const int32_t *text = ids + 3;
    const int n_text = n_ids - 8;
    // the role (3 rows), then tts_pad x (codec - 2) + tts_bos over the codec
    // ids but the last one
    for (int i = 0; i < 3; ++i) row(ids[i], -1);
    for (int i = 0; i < n_codec - 1; ++i) row(i < n_codec - 2 ? tok->tts_pad : tok->tts_bos, codec[i]);
    if (non_streaming) {
        // the text then tts_eos, each over codec_pad; tts_pad over codec_bos;
        // what follows is tts_pad alone
        for (int i = 0; i < n_text; ++i) row(text[i], tok->codec_pad);
        row(tok->tts_eos, tok->codec_pad);
        row(tok->tts_pad, tok->codec_bos);
        p.rows = static_cast<int>(p.text.size());
        row(tok->tts_pad, -1);
    } else {
        // the first text token over codec_bos; the next ones then tts_eos,
        // one per frame
        row(text[0], tok->codec_bos);
        p.rows = static_cast<int>(p.text.size());
        for (int i = 1; i < n_text; ++i) row(text[i], -1);
        row(tok->tts_eos, -1);
    }
    p.trailing = static_cast<int>(p.text.size()) - p.rows;
    row(tok->tts_pad, -1);
    return QTTS_OK;
}

// the rows, then the checks against the text projection and the talker
static int prompt_plan(const char *fn, const qtts_device *dev, int codec_vocab, const qtts_textproj *tp,
                       const qtts_prompt_tokens *tok, const int32_t *ids, int n_ids, const int32_t *codec, int n_codec,
                       int non_streaming, PromptPlan &p) {
    if (!tp) return set_err(QTTS_E_ARG, "%s: NULL argument", fn);
    int rc = plan_rows(fn, tok, ids, n_ids, codec, n_codec, non_streaming, p);
    if (rc) return rc;
    if (tp->dev != dev || tp->hidden != H)
        return set_err(QTTS_E_ARG, "%s: the text projection is on another device or %d wide", fn, tp->hidden);
    for (size_t r = 0; r < p.text.size(); ++r) {
        if (p.text[r] < 0 || p.text[r] >= tp->vocab)
            return set_err(QTTS_E_ARG, "%s: text token %d out of range", fn, p.text[r]);
        if (p.codec[r] >= codec_vocab) return set_err(QTTS_E_ARG, "%s: codec id %d out of range", fn, p.codec[r]);
        if (p.codec[r] < -1) return set_err(QTTS_E_ARG, "%s: codec id %d out of range", fn, p.codec[r]);
    }
    return QTTS_OK;
}

extern "C" int qtts_prompt_plan(const qtts_prompt_tokens *tok, const int32_t *ids, int n_ids, const int32_t *codec,
                                int n_codec, int non_streaming, int32_t *text_out, int32_t *codec_out, int cap,
                                int *rows, int *trailing_rows) {
    PromptPlan p;
    int rc = plan_rows("qtts_prompt_plan", tok, ids, n_ids, codec, n_codec, non_streaming, p);
    if (rc) return rc;
    if (rows) *rows = p.rows;
    if (trailing_rows) *trailing_rows = p.trailing;
    if (!text_out && !codec_out) return QTTS_OK;  // the counts alone
    const int n = p.rows + p.trailing;
    if (!text_out || !codec_out || cap < n)
        return set_err(QTTS_E_ARG, "qtts_prompt_plan: buffers of %d entries for %d rows", cap, n);
    memcpy(text_out, p.text.data(), static_cast<size_t>(n) * 4);
    memcpy(codec_out, p.codec.data(), static_cast<size_t>(n) * 4);
    return QTTS_OK;
}

extern "C" int qtts_talker_start_prompt(qtts_talker *t, qtts_textproj *tp, const qtts_prompt_tokens *tok,
                                        const int32_t *ids, int n_ids, const int32_t *codec, int n_codec,
                                        int non_streaming, float *logits, float *hidden) {
    if (!t) return set_err(QTTS_E_ARG, "qtts_talker_start_prompt: NULL talker");
    PromptPlan p;
    int rc = prompt_plan("qtts_talker_start_prompt", t->talker->dev, t->cfg.vocab, tp, tok, ids, n_ids, codec, n_codec,
                         non_streaming, p);
    if (rc) return rc;
    cudaStream_t st = t->talker->run.stream;
    rc = textproj_run(tp, p.text.data(), p.codec.data(), t->codec_emb, static_cast<int>(p.text.size()), st);
    if (rc) return rc;
    const float *y = tp->y;
    return talker_start(t, true, y, p.rows, y + static_cast<size_t>(p.rows) * H, p.trailing,
                        y + static_cast<size_t>(p.rows + p.trailing) * H, logits, hidden);
}

extern "C" int qtts_talker_prompt_rows(qtts_talker *t, qtts_textproj *tp, const qtts_prompt_tokens *tok,
                                       const int32_t *ids, int n_ids, const int32_t *codec, int n_codec,
                                       int non_streaming, float *prefill, int prefill_cap, float *trailing,
                                       int trailing_cap, int *rows, int *trailing_rows) {
    if (!t) return set_err(QTTS_E_ARG, "qtts_talker_prompt_rows: NULL talker");
    PromptPlan p;
    int rc = prompt_plan("qtts_talker_prompt_rows", t->talker->dev, t->cfg.vocab, tp, tok, ids, n_ids, codec, n_codec,
                         non_streaming, p);
    if (rc) return rc;
    if (rows) *rows = p.rows;
    if (trailing_rows) *trailing_rows = p.trailing;
    if (!prefill && !trailing) return QTTS_OK;  // the counts alone
    if (!prefill || !trailing || prefill_cap < p.rows || trailing_cap < p.trailing)
        return set_err(QTTS_E_ARG, "qtts_talker_prompt_rows: buffers of %d and %d rows for %d and %d", prefill_cap,
                       trailing_cap, p.rows, p.trailing);
    cudaStream_t st = t->talker->run.stream;
    rc = textproj_run(tp, p.text.data(), p.codec.data(), t->codec_emb, static_cast<int>(p.text.size()), st);
    if (rc) return rc;
    CK(cudaMemcpyAsync(prefill, tp->y, static_cast<size_t>(p.rows) * H * 4, cudaMemcpyDeviceToHost, st));
    if (p.trailing > 0)
        CK(cudaMemcpyAsync(trailing, tp->y + static_cast<size_t>(p.rows) * H, static_cast<size_t>(p.trailing) * H * 4,
                           cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return QTTS_OK;
}

extern "C" int qtts_textproj_destroy(qtts_textproj *t) {
    if (!t) return QTTS_OK;
    cudaSetDevice(t->dev->ordinal);
    textproj_free(t);
    return QTTS_OK;
}

// ------------------------------------------------------------------ files

struct qtts_safetensors {
    qtts_st::File f;
    std::string path;
};

extern "C" int qtts_safetensors_open(const char *path, qtts_safetensors **out) {
    if (!path || !out) return set_err(QTTS_E_ARG, "qtts_safetensors_open: NULL argument");
    *out = nullptr;
    qtts_safetensors *f = new qtts_safetensors();
    f->path = path;
    std::string err;
    if (!f->f.open(path, err)) {
        delete f;
        return set_err(QTTS_E_ARG, "qtts_safetensors_open: %s: %s", path, err.c_str());
    }
    *out = f;
    return QTTS_OK;
}

extern "C" int qtts_safetensors_count(qtts_safetensors *f, int *n) {
    if (!f || !n) return set_err(QTTS_E_ARG, "qtts_safetensors_count: NULL argument");
    *n = static_cast<int>(f->f.tensors.size());
    return QTTS_OK;
}

extern "C" int qtts_safetensors_name(qtts_safetensors *f, int i, char *buf, int len) {
    if (!f || !buf || len <= 0 || i < 0 || i >= static_cast<int>(f->f.tensors.size()))
        return set_err(QTTS_E_ARG, "qtts_safetensors_name: bad argument");
    const std::string &n = f->f.tensors[i].name;
    if (static_cast<int>(n.size()) >= len) return set_err(QTTS_E_ARG, "qtts_safetensors_name: buffer of %d for %d", len,
                                                          static_cast<int>(n.size()) + 1);
    memcpy(buf, n.c_str(), n.size() + 1);
    return QTTS_OK;
}

static int st_dtype(const std::string &d) {
    if (d == "F32") return QTTS_DTYPE_F32;
    if (d == "BF16") return QTTS_DTYPE_BF16;
    if (d == "F16") return QTTS_DTYPE_F16;
    return QTTS_DTYPE_OTHER;
}

extern "C" int qtts_safetensors_tensor(qtts_safetensors *f, const char *name, int *dtype, int *ndim, int64_t *shape,
                                       const void **data, int64_t *bytes) {
    if (!f || !name) return set_err(QTTS_E_ARG, "qtts_safetensors_tensor: NULL argument");
    const qtts_st::Tensor *t = f->f.find(name);
    if (!t) return set_err(QTTS_E_ARG, "qtts_safetensors_tensor: no tensor %s in %s", name, f->path.c_str());
    if (t->shape.size() > QTTS_MAX_DIMS)
        return set_err(QTTS_E_ARG, "qtts_safetensors_tensor: %s has %d dimensions", name,
                       static_cast<int>(t->shape.size()));
    if (dtype) *dtype = st_dtype(t->dtype);
    if (ndim) *ndim = static_cast<int>(t->shape.size());
    if (shape)
        for (size_t i = 0; i < t->shape.size(); ++i) shape[i] = t->shape[i];
    if (data) *data = f->f.data + t->begin;
    if (bytes) *bytes = static_cast<int64_t>(t->end - t->begin);
    return QTTS_OK;
}

extern "C" int qtts_safetensors_close(qtts_safetensors *f) {
    delete f;
    return QTTS_OK;
}

// the tensor `name` as [rows][cols] in F32 or BF16 (its bytes in the
// mapping), else QTTS_E_ARG as QwenWiden raises (lm.pas:164-168)
static int st_matrix(qtts_safetensors *f, const std::string &name, int64_t rows, int64_t cols, const void **data,
                     int *dtype) {
    const qtts_st::Tensor *t = f->f.find(name);
    if (!t) return set_err(QTTS_E_ARG, "%s: no tensor %s", f->path.c_str(), name.c_str());
    if (f->f.count(*t) != static_cast<uint64_t>(rows * cols))
        return set_err(QTTS_E_ARG, "%s: %s has %llu values instead of [%lld,%lld]", f->path.c_str(), name.c_str(),
                       static_cast<unsigned long long>(f->f.count(*t)), static_cast<long long>(rows),
                       static_cast<long long>(cols));
    const int dt = st_dtype(t->dtype);
    if (dt != QTTS_DTYPE_F32 && dt != QTTS_DTYPE_BF16)
        return set_err(QTTS_E_ARG, "%s: %s is %s (F32 or BF16 expected)", f->path.c_str(), name.c_str(),
                       t->dtype.c_str());
    *data = f->f.data + t->begin;
    *dtype = dt;
    return QTTS_OK;
}

// QwenWiden (lm.pas:159-172): the tensor widened to float32 on the host
static int st_widen(qtts_safetensors *f, const std::string &name, int64_t n, std::vector<float> &out) {
    const void *d;
    int dt;
    int rc = st_matrix(f, name, 1, n, &d, &dt);
    if (rc) return rc;
    out.resize(static_cast<size_t>(n));
    if (dt == QTTS_DTYPE_F32) {
        memcpy(out.data(), d, static_cast<size_t>(n) * 4);
    } else {
        const uint8_t *b = static_cast<const uint8_t *>(d);
        for (int64_t i = 0; i < n; ++i) {
            const uint32_t v = static_cast<uint32_t>(b[2 * i] | (b[2 * i + 1] << 8)) << 16;
            memcpy(&out[i], &v, 4);
        }
    }
    return QTTS_OK;
}

extern "C" int qtts_stack_create_safetensors(qtts_device *dev, const qtts_stack_config *c, qtts_safetensors *f,
                                             const char *prefix, qtts_stack **out) {
    if (!dev || !c || !f || !prefix || !out) return set_err(QTTS_E_ARG, "qtts_stack_create_safetensors: NULL argument");
    *out = nullptr;
    if (c->layers <= 0 || c->layers > 1024) return set_err(QTTS_E_ARG, "qtts_stack_create_safetensors: %d layers", c->layers);
    const int64_t hid = c->hidden, q = static_cast<int64_t>(c->heads) * c->head_dim,
                  kv = static_cast<int64_t>(c->kv_heads) * c->head_dim, inter = c->intermediate;
    std::vector<qtts_layer_src> src(c->layers);
    std::vector<std::vector<float>> norms(static_cast<size_t>(c->layers) * 4);
    for (int l = 0; l < c->layers; ++l) {
        const std::string p = std::string(prefix) + "layers." + std::to_string(l) + ".";
        qtts_layer_src &s = src[l];
        struct M {
            const char *name;
            int64_t rows, cols;
            const void **dst;
        } mats[] = {{"self_attn.q_proj.weight", q, hid, &s.q_proj},   {"self_attn.k_proj.weight", kv, hid, &s.k_proj},
                    {"self_attn.v_proj.weight", kv, hid, &s.v_proj},  {"self_attn.o_proj.weight", hid, q, &s.o_proj},
                    {"mlp.gate_proj.weight", inter, hid, &s.gate_proj}, {"mlp.up_proj.weight", inter, hid, &s.up_proj},
                    {"mlp.down_proj.weight", hid, inter, &s.down_proj}};
        for (int m = 0; m < 7; ++m) {
            int dt;
            int rc = st_matrix(f, p + mats[m].name, mats[m].rows, mats[m].cols, mats[m].dst, &dt);
            if (rc) return rc;
            if (m == 0) s.dtype = dt;
            if (dt != s.dtype)
                return set_err(QTTS_E_ARG, "%s: the matrices of layer %d mix F32 and BF16", f->path.c_str(), l);
        }
        const char *nn[4] = {"input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_norm.weight",
                             "self_attn.k_norm.weight"};
        const int64_t nl[4] = {hid, hid, c->head_dim, c->head_dim};
        for (int k = 0; k < 4; ++k) {
            int rc = st_widen(f, p + nn[k], nl[k], norms[static_cast<size_t>(l) * 4 + k]);
            if (rc) return rc;
        }
        s.input_norm = norms[static_cast<size_t>(l) * 4].data();
        s.post_norm = norms[static_cast<size_t>(l) * 4 + 1].data();
        s.q_norm = norms[static_cast<size_t>(l) * 4 + 2].data();
        s.k_norm = norms[static_cast<size_t>(l) * 4 + 3].data();
    }
    std::vector<float> fn;
    int rc = st_widen(f, std::string(prefix) + "norm.weight", hid, fn);
    if (rc) return rc;
    return qtts_stack_create(dev, c, src.data(), fn.data(), out);
}

extern "C" int qtts_heads_add_safetensors(qtts_heads *h, qtts_safetensors *f, const char *name, int rows, int *index) {
    if (!h || !f || !name) return set_err(QTTS_E_ARG, "qtts_heads_add_safetensors: NULL argument");
    if (rows <= 0) return set_err(QTTS_E_ARG, "qtts_heads_add_safetensors: %d rows", rows);
    const void *d;
    int dt;
    int rc = st_matrix(f, name, rows, h->hidden, &d, &dt);
    if (rc) return rc;
    return qtts_heads_add(h, d, dt, rows, index);
}

// The cached blob of a stack: its weights in the device format (F32 rows or
// row-packed Q8_0, as held), written and read back without a conversion.
//   "QTTSSTK1" | qtts_stack_config | per layer: wqkv wo wgu wd (device
//   bytes), input / post / q / k norms (float32) | final norm | crc32c of
//   all the bytes before it (u32, little-endian)
static const char BLOB_MAGIC[8] = {'Q', 'T', 'T', 'S', 'S', 'T', 'K', '1'};

struct LayerBytes {
    size_t qkv, o, gu, d;
};
static LayerBytes layer_bytes(int wdt) {
    return {static_cast<size_t>(QKV_ROWS) * row_bytes(wdt, H), static_cast<size_t>(H) * row_bytes(wdt, QDIM),
            static_cast<size_t>(GU_ROWS) * row_bytes(wdt, H), static_cast<size_t>(H) * row_bytes(wdt, INTER)};
}

extern "C" int qtts_stack_save(const qtts_stack *s, const char *path) {
    if (!s || !path) return set_err(QTTS_E_ARG, "qtts_stack_save: NULL argument");
    CK(cudaSetDevice(s->dev->ordinal));
    const int wdt = s->cfg.dtype == QTTS_DTYPE_F32 ? WDT_F32 : WDT_Q8;
    const LayerBytes lb = layer_bytes(wdt);
    std::vector<uint8_t> blob(sizeof(BLOB_MAGIC) + sizeof(qtts_stack_config));
    memcpy(blob.data(), BLOB_MAGIC, sizeof(BLOB_MAGIC));
    memcpy(blob.data() + sizeof(BLOB_MAGIC), &s->cfg, sizeof(qtts_stack_config));
    auto append = [&](const void *dptr, size_t n) -> int {
        const size_t at = blob.size();
        blob.resize(at + n);
        CK(cudaMemcpy(blob.data() + at, dptr, n, cudaMemcpyDeviceToHost));
        return QTTS_OK;
    };
    int rc = QTTS_OK;
    for (const DLayer &d : s->hlayers) {
        if ((rc = append(d.wqkv, lb.qkv)) || (rc = append(d.wo, lb.o)) || (rc = append(d.wgu, lb.gu)) ||
            (rc = append(d.wd, lb.d)) || (rc = append(d.in_norm, H * 4)) || (rc = append(d.post_norm, H * 4)) ||
            (rc = append(d.q_norm, HD * 4)) || (rc = append(d.k_norm, HD * 4)))
            return rc;
    }
    if ((rc = append(s->d_final_norm, H * 4))) return rc;
    const uint32_t crc = crc32c(0, blob.data(), blob.size());
    for (int i = 0; i < 4; ++i) blob.push_back(static_cast<uint8_t>(crc >> (8 * i)));
    const std::string tmp = std::string(path) + ".tmp";
    FILE *fp = fopen(tmp.c_str(), "wb");
    if (!fp) return set_err(QTTS_E_ARG, "qtts_stack_save: cannot write %s", tmp.c_str());
    const bool ok = fwrite(blob.data(), 1, blob.size(), fp) == blob.size();
    if (fclose(fp) != 0 || !ok || rename(tmp.c_str(), path) != 0) {
        remove(tmp.c_str());
        return set_err(QTTS_E_ARG, "qtts_stack_save: writing %s failed", path);
    }
    return QTTS_OK;
}

extern "C" int qtts_stack_load(qtts_device *dev, const char *path, qtts_stack **out) {
    if (!dev || !path || !out) return set_err(QTTS_E_ARG, "qtts_stack_load: NULL argument");
    *out = nullptr;
    qtts_st::File map;  // only its mapping is used
    map.fd = ::open(path, O_RDONLY | O_CLOEXEC);
    struct stat st;
    if (map.fd < 0 || fstat(map.fd, &st) != 0) return set_err(QTTS_E_ARG, "qtts_stack_load: cannot open %s", path);
    map.size = static_cast<size_t>(st.st_size);
    const size_t head = sizeof(BLOB_MAGIC) + sizeof(qtts_stack_config);
    if (map.size < head + 4) return set_err(QTTS_E_ARG, "qtts_stack_load: %s is no stack blob", path);
    map.map = mmap(nullptr, map.size, PROT_READ, MAP_PRIVATE, map.fd, 0);
    if (map.map == MAP_FAILED) {
        map.map = nullptr;
        return set_err(QTTS_E_ARG, "qtts_stack_load: mmap of %s failed", path);
    }
    const uint8_t *b = static_cast<const uint8_t *>(map.map);
    qtts_stack_config c;
    memcpy(&c, b + sizeof(BLOB_MAGIC), sizeof(c));
    if (memcmp(b, BLOB_MAGIC, sizeof(BLOB_MAGIC)) != 0 || !dims_ok(&c) || c.layers > 1024 ||
        (c.dtype != QTTS_DTYPE_F32 && c.dtype != QTTS_DTYPE_Q8_0))
        return set_err(QTTS_E_ARG, "qtts_stack_load: %s is no stack blob of this build's dimensions", path);
    const int wdt = c.dtype == QTTS_DTYPE_F32 ? WDT_F32 : WDT_Q8;
    const LayerBytes lb = layer_bytes(wdt);
    const size_t per_layer = lb.qkv + lb.o + lb.gu + lb.d + (2 * H + 2 * HD) * 4;
    if (map.size != head + per_layer * c.layers + H * 4 + 4)
        return set_err(QTTS_E_ARG, "qtts_stack_load: %s has %zu bytes, %zu expected", path, map.size,
                       head + per_layer * c.layers + H * 4 + 4);
    uint32_t want = 0;
    for (int i = 3; i >= 0; --i) want = (want << 8) | b[map.size - 4 + i];
    if (crc32c(0, b, map.size - 4) != want) return set_err(QTTS_E_ARG, "qtts_stack_load: %s: checksum mismatch", path);
    // the layers from their device bytes, uploaded as they are; then the
    // create path's norms, per-head layouts and layer table
    struct BlobFill : LayerFill {
        const uint8_t *base;
        LayerBytes lb;
        size_t per_layer;
        int matrices(int l, uint8_t *wqkv, uint8_t *wo, uint8_t *wgu, uint8_t *wd) override {
            const uint8_t *p = base + per_layer * l;
            CK(cudaMemcpy(wqkv, p, lb.qkv, cudaMemcpyHostToDevice));
            CK(cudaMemcpy(wo, p + lb.qkv, lb.o, cudaMemcpyHostToDevice));
            CK(cudaMemcpy(wgu, p + lb.qkv + lb.o, lb.gu, cudaMemcpyHostToDevice));
            CK(cudaMemcpy(wd, p + lb.qkv + lb.o + lb.gu, lb.d, cudaMemcpyHostToDevice));
            return QTTS_OK;
        }
        void norms(int l, const float *n[4]) override {
            const uint8_t *p = base + per_layer * l + lb.qkv + lb.o + lb.gu + lb.d;
            n[0] = reinterpret_cast<const float *>(p);
            n[1] = reinterpret_cast<const float *>(p + H * 4);
            n[2] = reinterpret_cast<const float *>(p + 2 * H * 4);
            n[3] = reinterpret_cast<const float *>(p + 2 * H * 4 + HD * 4);
        }
    } fill;
    fill.base = b + head;
    fill.lb = lb;
    fill.per_layer = per_layer;
    return stack_build(dev, &c, fill, reinterpret_cast<const float *>(b + head + per_layer * c.layers), out);
}

extern "C" int qtts_quantize_q8_0(qtts_device *dev, const float *src, int64_t n, uint8_t *dst) {
    if (!dev || !src || !dst || n < 0 || (n & 31) != 0) return set_err(QTTS_E_ARG, "qtts_quantize_q8_0: bad argument");
    if (n == 0) return QTTS_OK;
    CK(cudaSetDevice(dev->ordinal));
    float *d_src = nullptr;
    uint8_t *d_dst = nullptr;
    long long nb = n / 32;
    CK(cudaMalloc(&d_src, n * 4));
    cudaError_t e = cudaMalloc(&d_dst, nb * 34);
    if (e != cudaSuccess) {
        cudaFree(d_src);
        return set_err(QTTS_E_OOM, "qtts_quantize_q8_0: %s", cudaGetErrorString(e));
    }
    int rc = QTTS_OK;
    if (cudaMemcpy(d_src, src, n * 4, cudaMemcpyHostToDevice) != cudaSuccess) rc = set_err(QTTS_E_CUDA, "upload failed");
    if (rc == QTTS_OK) {
        quantize_ggml_kernel<<<static_cast<unsigned>((nb + 255) / 256), 256, 0, dev->load>>>(d_src, nb, d_dst);
        if (cudaStreamSynchronize(dev->load) != cudaSuccess ||
            cudaMemcpy(dst, d_dst, nb * 34, cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = set_err(QTTS_E_CUDA, "qtts_quantize_q8_0: %s", cudaGetErrorString(cudaGetLastError()));
    }
    cudaFree(d_src);
    cudaFree(d_dst);
    return rc;
}

// ------------------------------------------------------------------ forward without allocation
//
// qtts_lm_forward_noalloc: the same forward as qtts_lm_forward, for callers
// that must not allocate device memory while they run it -- a real-time
// synthesis thread, for which cudaMalloc/cudaFree (which can synchronise the
// whole device and block for milliseconds) is off limits, or a host
// application whose GPU memory is all handed out by its own pool allocator.
// Inputs and outputs are the caller's device buffers; the kernel's scratch
// (residual rows, q/k/v, SwiGLU activations, attention partials, argmax keys,
// barrier and error words) lives in one static device array instead of
// buffers of the lm.  Limits: a grid of at most NOALLOC_MAX_SMS CTAs (one per
// SM) and heads of at most NOALLOC_MAX_HEAD_ROWS rows.

constexpr int NOALLOC_MAX_SMS = 160;
constexpr int NOALLOC_MAX_HEAD_ROWS = 4096;

namespace {
constexpr size_t al256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }
constexpr size_t NA_X = 0;
constexpr size_t NA_X8 = NA_X + al256(static_cast<size_t>(RMAX) * H * 4);
constexpr size_t NA_QKV = NA_X8 + al256(static_cast<size_t>(RMAX) * H * 8);
constexpr size_t NA_ACT = NA_QKV + al256(static_cast<size_t>(RMAX) * QKV_ROWS * 8);
constexpr size_t NA_PART = NA_ACT + al256(static_cast<size_t>(RMAX) * INTER * 4);
constexpr size_t NA_ARG =
    NA_PART + al256(static_cast<size_t>(HKV) * (NOALLOC_MAX_SMS / HKV) * RMAX * 2 * PSTRIDE * 4);
constexpr size_t NA_BAR = NA_ARG + al256(static_cast<size_t>(NOALLOC_MAX_SMS) * 8);
constexpr size_t NA_ERR = NA_BAR + al256(BAR_WORDS * 4);
constexpr size_t NA_LOGITS = NA_ERR + al256(16);
constexpr size_t NA_HIDDEN = NA_LOGITS + al256(static_cast<size_t>(NOALLOC_MAX_HEAD_ROWS) * 4);
constexpr size_t NA_XT = NA_HIDDEN + al256(H * 4);
constexpr size_t NA_BYTES = NA_XT + al256(H * 4);  // 931,584 bytes
}  // namespace

// Every GPU that loads the library holds this array until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[NA_BYTES];

// its device address, per device (taken once, with that device current:
// by qtts_lm_create, or else by the first call on the device)
static std::mutex g_noalloc_mu;
static void *g_noalloc_ptr[256];
static unsigned g_noalloc_epoch[256];  // launch epoch of the array's tagged words, per device

static void *noalloc_lookup(int ordinal) {
    if (ordinal < 0 || ordinal >= 256) return nullptr;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[ordinal]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) == cudaSuccess && p) g_noalloc_ptr[ordinal] = p;
    }
    return g_noalloc_ptr[ordinal];
}

static int noalloc_scratch(int ordinal, unsigned char **out) {
    if (ordinal < 0 || ordinal >= 256) return set_err(QTTS_E_ARG, "qtts_lm_forward_noalloc: device %d", ordinal);
    void *p = noalloc_lookup(ordinal);
    if (!p) {
        void *q = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&q, g_noalloc_scratch);
        return set_err(QTTS_E_CUDA, "qtts_lm_forward_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    }
    *out = static_cast<unsigned char *>(p);
    return QTTS_OK;
}

extern "C" int qtts_lm_forward_noalloc(qtts_lm *m, const float *x, int rows, int head, float *logits,
                                       float *hidden) {
    if (!m) return set_err(QTTS_E_ARG, "qtts_lm_forward_noalloc: NULL lm");
    if (rows <= 0) return QTTS_OK;
    if (!x) return set_err(QTTS_E_ARG, "qtts_lm_forward_noalloc: x is NULL");
    // the kernel moves these rows with 16-byte loads and stores: an address
    // off that boundary is refused here, before anything is launched
    const auto off16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; };
    if (off16(x) || (logits && off16(logits)) || (hidden && off16(hidden)))
        return set_err(QTTS_E_ARG, "qtts_lm_forward_noalloc: x, logits and hidden must be 16-byte aligned");
    if (logits && (head < 0 || head >= static_cast<int>(m->heads->mats.size())))
        return set_err(QTTS_E_ARG, "qtts_lm_forward_noalloc: no head %d in %s", head, m->heads->name.c_str());
    if (logits && m->heads->mats[head].rows > NOALLOC_MAX_HEAD_ROWS)
        return set_err(QTTS_E_CAPACITY, "qtts_lm_forward_noalloc: head of %d rows, the static scratch holds %d",
                       m->heads->mats[head].rows, NOALLOC_MAX_HEAD_ROWS);
    if (m->dev->sms > NOALLOC_MAX_SMS)
        return set_err(QTTS_E_CAPACITY, "qtts_lm_forward_noalloc: a grid of %d CTAs, the static scratch holds %d",
                       m->dev->sms, NOALLOC_MAX_SMS);
    if (m->len + rows > m->max_pos)
        return set_err(QTTS_E_CAPACITY, "qtts_lm_forward_noalloc: %d + %d positions, the cache holds %d", m->len,
                       rows, m->max_pos);
    CK(cudaSetDevice(m->dev->ordinal));
    unsigned char *sc = nullptr;
    int rc = noalloc_scratch(m->dev->ordinal, &sc);
    if (rc) return rc;
    Runner r;
    r.stream = m->run.stream;
    r.grid = m->dev->sms;
    r.block = nullptr;
    r.h_err = nullptr;
    r.s.x = reinterpret_cast<float *>(sc + NA_X);
    r.s.x8 = reinterpret_cast<unsigned long long *>(sc + NA_X8);
    r.s.qkv = reinterpret_cast<unsigned long long *>(sc + NA_QKV);
    // the array's tagged words and their epoch live as long as the array
    r.epoch = &g_noalloc_epoch[m->dev->ordinal];
    r.s.act = reinterpret_cast<float *>(sc + NA_ACT);
    r.s.part = reinterpret_cast<float *>(sc + NA_PART);
    r.s.arg = reinterpret_cast<unsigned long long *>(sc + NA_ARG);
    r.s.bar = reinterpret_cast<unsigned *>(sc + NA_BAR);
    r.s.err = reinterpret_cast<int *>(sc + NA_ERR);
    r.s.logits = logits ? logits : reinterpret_cast<float *>(sc + NA_LOGITS);
    r.s.hidden = hidden ? hidden : reinterpret_cast<float *>(sc + NA_HIDDEN);
    r.s.xt = reinterpret_cast<float *>(sc + NA_XT);
    // the array keeps the last call's contents: the barrier counters and the
    // error word must start at zero
    CK(cudaMemsetAsync(r.s.bar, 0, BAR_WORDS * 4, r.stream));
    CK(cudaMemsetAsync(r.s.err, 0, 16, r.stream));
    const int wdt = m->stack->cfg.dtype == QTTS_DTYPE_F32 ? WDT_F32 : WDT_Q8;
    Job j = base_job(m);
    j.s = r.s;
    j.mode = 0;
    j.st = dstack(m->stack);
    j.ctx.k = m->k;
    j.ctx.v = m->v;
    j.ctx.kv16 = m->kv16;
    j.ctx.max_pos = m->max_pos;
    for (int r0 = 0; r0 < rows; r0 += RMAX) {
        const int n = rows - r0 < RMAX ? rows - r0 : RMAX;
        const bool last = r0 + n == rows;
        j.xin = x + static_cast<size_t>(r0) * H;  // the caller's rows, read in place
        j.rows = n;
        j.L0 = m->len;
        j.head_w = (last && logits) ? m->heads->mats[head].d : nullptr;
        j.head_rows = (last && logits) ? m->heads->mats[head].rows : 0;
        rc = launch(m->dev, r, j, wdt);
        if (rc) return rc;
        int err[2] = {0, 0};
        CK(cudaMemcpyAsync(err, r.s.err, 8, cudaMemcpyDeviceToHost, r.stream));
        CK(cudaStreamSynchronize(r.stream));
        if (err[0] != 0) {
            CK(cudaMemsetAsync(r.s.bar, 0, BAR_WORDS * 4, r.stream));
            CK(cudaMemsetAsync(r.s.err, 0, 16, r.stream));
            CK(cudaStreamSynchronize(r.stream));
            return set_err(err[0] == ERR_CAPACITY ? QTTS_E_CAPACITY : QTTS_E_TIMEOUT,
                           "qtts_lm_forward_noalloc: device wait gave up (code %d at %d)", err[0], err[1]);
        }
        m->len += n;
    }
    return QTTS_OK;
}


// ------------------------------------------------------------------ batched forward
//
// qtts_batch: one stack (not owned) run for many sequences at once -- the
// TQwenLm.Forward protocol (lm.pas:391-408) for a batch of utterances, with a
// paged KV cache and the projections on the tcgen05 GEMM.

struct qtts_batch {
    qtts_device *dev;
    qtts_stack *stack;
    qtts_heads *heads;
    int max_seqs, max_tokens, max_pos, kv_dtype, mpps, npages, head_rows;
    void *pool;
    __half *kv16;  // the fp16 mirror of the pages (tensor-core prefill attention), or NULL
    int *d_pages;
    std::vector<int> h_pages;  // [max_seqs][mpps], -1 = none
    std::vector<int> free_pages;
    std::vector<int> len;
    float *rope_cos, *rope_sin;
    cudaStream_t stream;
    // per-call buffers
    float *x, *q32, *part, *hidden, *logits;
    __half *h16, *attn16, *act16, *hlast16;
    int *meta;  // token metadata and attention items
    size_t meta_bytes;
    int *err;
    std::vector<void *> allocs;
    // pinned staging of the per-call metadata and page table: a ring, so
    // that the host builds call k+1 while call k's copy is still queued
    static constexpr int NSLOT = 4;
    int *hmeta[NSLOT] = {};
    cudaEvent_t mev[NSLOT] = {};
    bool mev_live[NSLOT] = {};
    int mslot = 0;
    // fixed pinned slots, one per call of a frame graph (read by its copies)
    static constexpr int NFIXED = 16;
    int *hfixed[NFIXED] = {};
    size_t max_parts = 0;  // attention partials the part buffer holds
};

static void batch_free(qtts_batch *b) {
    for (int k = 0; k < qtts_batch::NSLOT; ++k) {
        if (b->mev[k]) cudaEventDestroy(b->mev[k]);
        if (b->hmeta[k]) cudaFreeHost(b->hmeta[k]);
    }
    for (int k = 0; k < qtts_batch::NFIXED; ++k)
        if (b->hfixed[k]) cudaFreeHost(b->hfixed[k]);
    for (void *p : b->allocs) cudaFree(p);
    if (b->stream) cudaStreamDestroy(b->stream);
    delete b;
}

extern "C" int qtts_batch_create(qtts_stack *stack, qtts_heads *heads, int max_seqs, int max_tokens, int max_pos,
                                 int kv_dtype, qtts_batch **out) {
    if (!stack || !heads || !out) return set_err(QTTS_E_ARG, "qtts_batch_create: NULL argument");
    *out = nullptr;
    if (max_seqs <= 0 || max_tokens <= 0 || max_pos <= 0 || max_tokens < max_seqs)
        return set_err(QTTS_E_ARG, "qtts_batch_create: bad sizes (%d seqs, %d tokens, %d positions)", max_seqs,
                       max_tokens, max_pos);
    if (kv_dtype != QTTS_DTYPE_F32 && kv_dtype != QTTS_DTYPE_BF16)
        return set_err(QTTS_E_ARG, "qtts_batch_create: KV cache in F32 or BF16");
    if (heads->hidden != stack->cfg.hidden || heads->dtype != stack->cfg.dtype)
        return set_err(QTTS_E_ARG, "qtts_batch_create: heads and stack do not match");
    qtts_device *dev = stack->dev;
    CK(cudaSetDevice(dev->ordinal));
    int rc0 = gemm_init(dev);
    if (rc0 == QTTS_OK) rc0 = stack_tiles(stack);
    if (rc0 == QTTS_OK) rc0 = heads_tiles(heads);
    if (rc0) return rc0;
    qtts_batch *b = new qtts_batch();
    b->dev = dev;
    b->stack = stack;
    b->heads = heads;
    b->max_seqs = max_seqs;
    b->max_tokens = max_tokens;
    b->max_pos = max_pos;
    b->kv_dtype = kv_dtype;
    b->mpps = (max_pos + PAGE - 1) / PAGE;
    b->npages = max_seqs * b->mpps;
    b->head_rows = 0;
    for (const HeadMat &m : heads->mats) b->head_rows = m.rows > b->head_rows ? m.rows : b->head_rows;
    b->h_pages.assign(static_cast<size_t>(max_seqs) * b->mpps, -1);
    for (int p = b->npages - 1; p >= 0; --p) b->free_pages.push_back(p);
    b->len.assign(max_seqs, 0);
    const int L = stack->cfg.layers;
    const size_t kvb = kv_dtype == QTTS_DTYPE_F32 ? 4 : 2;
    const size_t T = max_tokens;
    const int max_splits = std::max((max_pos + DSPLIT - 1) / DSPLIT, DMAX_SPLITS);
    const int max_items = max_tokens * HKV + max_seqs * HKV * max_splits;
    b->max_parts = static_cast<size_t>(max_seqs) * HKV * max_splits;
    b->meta_bytes = (T * 2 + static_cast<size_t>(max_items) * (sizeof(AttnItem) / 4) + max_seqs * (HKV * 2 + 2)) * 4;
    struct A {
        void **p;
        size_t bytes;
    } want[] = {
        {&b->pool, static_cast<size_t>(b->npages) * L * 2 * HKV * PAGE * HD * kvb},
        {reinterpret_cast<void **>(&b->d_pages), b->h_pages.size() * 4},
        {reinterpret_cast<void **>(&b->rope_cos), static_cast<size_t>(max_pos) * (HD / 2) * 4},
        {reinterpret_cast<void **>(&b->rope_sin), static_cast<size_t>(max_pos) * (HD / 2) * 4},
        {reinterpret_cast<void **>(&b->x), T * H * 4},
        {reinterpret_cast<void **>(&b->q32), T * QDIM * 4},
        {reinterpret_cast<void **>(&b->part), static_cast<size_t>(max_seqs) * HKV * max_splits * 2 * PSTRIDE * 4},
        {reinterpret_cast<void **>(&b->hidden), static_cast<size_t>(max_seqs) * H * 4},
        {reinterpret_cast<void **>(&b->logits), static_cast<size_t>(max_seqs) * (b->head_rows > 0 ? b->head_rows : 1) * 4},
        {reinterpret_cast<void **>(&b->h16), T * H * 2},
        {reinterpret_cast<void **>(&b->attn16), T * QDIM * 2},
        {reinterpret_cast<void **>(&b->act16), T * INTER * 2},
        {reinterpret_cast<void **>(&b->hlast16), static_cast<size_t>(max_seqs) * H * 2},
        {reinterpret_cast<void **>(&b->meta), b->meta_bytes},
        {reinterpret_cast<void **>(&b->err), 16},
    };
    for (const A &a : want) {
        if (cudaMalloc(a.p, a.bytes) != cudaSuccess) {
            batch_free(b);
            return set_err(QTTS_E_OOM, "qtts_batch_create: out of device memory (%zu bytes)", a.bytes);
        }
        b->allocs.push_back(*a.p);
    }
    std::vector<float> cs, sn;
    rope_tables(max_pos, stack->cfg.rope_theta, cs, sn);
    if (cudaMemcpy(b->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(b->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(b->err, 0, 16) != cudaSuccess ||
        cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking) != cudaSuccess) {
        batch_free(b);
        return set_err(QTTS_E_CUDA, "qtts_batch_create: set-up failed");
    }
    // a batch that can take long runs of new rows keeps the fp16 mirror of
    // its pages for the tensor-core attention (cleared: a page's unwritten
    // rows enter the P V product with weight 0 and must hold no NaN)
    if (max_tokens > TC_MIN_ROWS) {
        const size_t bytes = static_cast<size_t>(b->npages) * L * 2 * HKV * KV16_PAGE;
        if (cudaMalloc(&b->kv16, bytes) != cudaSuccess) {
            b->kv16 = nullptr;
            batch_free(b);
            return set_err(QTTS_E_OOM, "qtts_batch_create: out of device memory (%zu bytes)", bytes);
        }
        b->allocs.push_back(b->kv16);
        if (cudaMemsetAsync(b->kv16, 0, bytes, b->stream) != cudaSuccess ||
            cudaStreamSynchronize(b->stream) != cudaSuccess) {
            batch_free(b);
            return set_err(QTTS_E_CUDA, "qtts_batch_create: set-up failed");
        }
    }
    for (int k = 0; k < qtts_batch::NSLOT; ++k) {
        if (cudaHostAlloc(reinterpret_cast<void **>(&b->hmeta[k]), b->meta_bytes + b->h_pages.size() * 4,
                          cudaHostAllocDefault) != cudaSuccess ||
            cudaEventCreateWithFlags(&b->mev[k], cudaEventDisableTiming) != cudaSuccess) {
            batch_free(b);
            return set_err(QTTS_E_OOM, "qtts_batch_create: out of pinned host memory");
        }
    }
    *out = b;
    return QTTS_OK;
}

extern "C" int qtts_batch_reset(qtts_batch *b, int seq) {
    if (!b || seq < 0 || seq >= b->max_seqs) return set_err(QTTS_E_ARG, "qtts_batch_reset: bad sequence %d", seq);
    for (int i = 0; i < b->mpps; ++i) {
        int &pg = b->h_pages[static_cast<size_t>(seq) * b->mpps + i];
        if (pg >= 0) b->free_pages.push_back(pg);
        pg = -1;
    }
    b->len[seq] = 0;
    return QTTS_OK;
}

extern "C" int qtts_batch_length(qtts_batch *b, int seq, int *length) {
    if (!b || !length || seq < 0 || seq >= b->max_seqs) return set_err(QTTS_E_ARG, "qtts_batch_length: bad argument");
    *length = b->len[seq];
    return QTTS_OK;
}

// blocks of rmsnorm_f16_kernel: 8 rows (warps) each
static unsigned norm_grid(int rows) { return static_cast<unsigned>((rows + 7) / 8); }

template <class KVT>
static void batch_layers(qtts_batch *b, int T, int npitems, const AttnItem *pitems, int nditems,
                         const AttnItem *ditems, int ntitems, const AttnItem *titems, const int *tok_seq,
                         const int *tok_pos, int ncomb, const int *cfirst, const int *ccount, const int *ctok, int wdt,
                         cudaStream_t st, int &rc) {
    const qtts_stack *s = b->stack;
    KVPool<KVT> pool;
    pool.base = static_cast<KVT *>(b->pool);
    pool.pages = b->d_pages;
    pool.mpps = b->mpps;
    pool.layers = s->cfg.layers;
    const float eps = s->cfg.rms_eps;
    const int cap = b->max_tokens;
    for (int l = 0; l < s->cfg.layers && rc == QTTS_OK; ++l) {
        const DLayer &Ly = s->tlayers[l];
        cudaError_t e = launch_pdl(rmsnorm_f16_kernel, dim3(norm_grid(T)), dim3(256), 0, st, b->x, nullptr, T,
                                   Ly.in_norm, eps, b->h16, static_cast<float *>(nullptr));
        if (e != cudaSuccess) {
            rc = set_err(QTTS_E_CUDA, "qtts_batch_forward: launch failed: %s", cudaGetErrorString(e));
            return;
        }
        // the QKV GEMM's epilogue does q/k-norm + RoPE + the append to the pages
        QkvEpi qe;
        qe.q32 = b->q32;
        qe.q_norm = Ly.q_norm;
        qe.k_norm = Ly.k_norm;
        qe.rope_cos = b->rope_cos;
        qe.rope_sin = b->rope_sin;
        qe.eps = eps;
        qe.tok_seq = tok_seq;
        qe.tok_pos = tok_pos;
        qe.kv_base = pool.base;
        qe.kv_pages = pool.pages;
        qe.kv_mpps = pool.mpps;
        qe.kv_layers = pool.layers;
        qe.kv_layer = l;
        qe.kv_bf16 = sizeof(KVT) == 2 ? 1 : 0;
        qe.kv16 = b->kv16;
        if ((rc = gemm(Ly.wqkv, wdt, QKV_ROWS, H, b->h16, T, cap, nullptr, QKV_ROWS, false, b->err, st, nullptr, &qe)))
            return;
        if (npitems > 0)
            e = launch_pdl(attn_kernel<KVT>, dim3(npitems), dim3(ATHREADS), 0, st, pitems, b->q32, pool, l, b->attn16);
        if (e == cudaSuccess && ntitems > 0)
            e = launch_pdl(attn_prefill_tc_kernel<KVT>, dim3(ntitems), dim3(TA_THREADS), sizeof(TaSmem) + 1024, st,
                           titems, static_cast<const float *>(b->q32), pool, static_cast<const __half *>(b->kv16), l,
                           b->attn16, b->err);
        if (e == cudaSuccess && nditems > 0)
            e = launch_pdl(attn_decode_kernel<KVT>, dim3(nditems), dim3(DTHREADS), sizeof(DecodeSmem<KVT>), st, ditems,
                           b->q32, pool, l, b->attn16, b->part, b->err);
        if (e == cudaSuccess && ncomb > 0)
            e = launch_pdl(attn_combine_kernel, dim3((ncomb * HQ + 7) / 8), dim3(256), 0, st, cfirst, ccount, ctok,
                           ncomb, static_cast<const float *>(b->part), b->attn16);
        if (e != cudaSuccess) {
            rc = set_err(QTTS_E_CUDA, "qtts_batch_forward: launch failed: %s", cudaGetErrorString(e));
            return;
        }
        if ((rc = gemm(Ly.wo, wdt, H, QDIM, b->attn16, T, cap, b->x, H, true, b->err, st))) return;
        e = launch_pdl(rmsnorm_f16_kernel, dim3(norm_grid(T)), dim3(256), 0, st, b->x, nullptr, T, Ly.post_norm,
                       eps, b->h16, static_cast<float *>(nullptr));
        if (e != cudaSuccess) {
            rc = set_err(QTTS_E_CUDA, "qtts_batch_forward: launch failed: %s", cudaGetErrorString(e));
            return;
        }
        if ((rc = gemm(Ly.wgu, wdt, GU_ROWS, H, b->h16, T, cap, nullptr, INTER, false, b->err, st, b->act16)))
            return;
        if ((rc = gemm(Ly.wd, wdt, H, INTER, b->act16, T, cap, b->x, H, true, b->err, st))) return;
    }
    if (rc == QTTS_OK && cudaGetLastError() != cudaSuccess)
        rc = set_err(QTTS_E_CUDA, "qtts_batch_forward: kernel launch failed");
}

// The host half of one batched forward: validation, KV pages, the token
// metadata and attention items, staged in pinned memory (a slot of the ring,
// or the fixed slot `fixed` of the frame graphs); b->len advances.  Decode
// rows (one new row of a sequence) get `dsplits` page-aligned context splits
// each (0: one split per DSPLIT keys).
struct BatchPlan {
    int nseq, T, np, nd, ntc, ncomb, ring;  // ring: slot of the ring, -1 = fixed slot
    size_t meta_ints, o_ditems, o_titems, o_cf, o_cc, o_ct, o_last;
    const int *hm;                     // pinned: meta | page table
    bool same_shape(const BatchPlan &o) const {
        return nseq == o.nseq && T == o.T && np == o.np && nd == o.nd && ntc == o.ntc && ncomb == o.ncomb &&
               meta_ints == o.meta_ints && hm == o.hm;
    }
};

static int batch_plan(qtts_batch *b, int nseq, const int32_t *seqs, const int32_t *rows, int dsplits, int fixed,
                      BatchPlan *P) {
    if (!b || nseq <= 0 || !seqs || !rows) return set_err(QTTS_E_ARG, "qtts_batch_forward: bad argument");
    if (nseq > b->max_seqs) return set_err(QTTS_E_ARG, "qtts_batch_forward: %d sequences, at most %d", nseq, b->max_seqs);
    if (dsplits < 0 || dsplits > DMAX_SPLITS) return set_err(QTTS_E_ARG, "qtts_batch_forward: %d splits", dsplits);
    // validate, count tokens, allocate pages
    int T = 0;
    std::vector<char> seen(b->max_seqs, 0);
    for (int i = 0; i < nseq; ++i) {
        const int sq = seqs[i], n = rows[i];
        if (sq < 0 || sq >= b->max_seqs || seen[sq] || n <= 0)
            return set_err(QTTS_E_ARG, "qtts_batch_forward: entry %d (sequence %d, %d rows)", i, sq, n);
        seen[sq] = 1;
        if (b->len[sq] + n > b->max_pos)
            return set_err(QTTS_E_CAPACITY, "qtts_batch_forward: sequence %d: %d + %d positions, at most %d", sq,
                           b->len[sq], n, b->max_pos);
        T += n;
    }
    if (T > b->max_tokens) return set_err(QTTS_E_CAPACITY, "qtts_batch_forward: %d rows, at most %d", T, b->max_tokens);
    for (int i = 0; i < nseq; ++i) {
        const int sq = seqs[i];
        const int need = (b->len[sq] + rows[i] + PAGE - 1) / PAGE;
        for (int pg = 0; pg < need; ++pg) {
            int &slot = b->h_pages[static_cast<size_t>(sq) * b->mpps + pg];
            if (slot < 0) {
                if (b->free_pages.empty()) return set_err(QTTS_E_CAPACITY, "qtts_batch_forward: out of KV pages");
                slot = b->free_pages.back();
                b->free_pages.pop_back();
            }
        }
    }
    // metadata: tokens, attention items, combine lists
    std::vector<int> tok_seq(T), tok_pos(T), last(nseq);
    std::vector<AttnItem> pitems, ditems, titems;
    std::vector<int> cfirst, ccount, ctok;
    int t = 0, nparts = 0;
    for (int i = 0; i < nseq; ++i) {
        const int sq = seqs[i], n = rows[i], L0 = b->len[sq];
        for (int r = 0; r < n; ++r) {
            tok_seq[t + r] = sq;
            tok_pos[t + r] = L0 + r;
        }
        last[i] = t + n - 1;
        if (n == 1) {
            // one query: page-aligned splits of the context, combined
            // afterwards when there are several (a split may be empty)
            const int ctx = L0 + 1;
            const int S = dsplits > 0 ? dsplits : (ctx + DSPLIT - 1) / DSPLIT;
            for (int h = 0; h < HKV; ++h) {
                if (S > 1) {
                    cfirst.push_back(nparts);
                    ccount.push_back(S);
                }
                for (int sp = 0; sp < S; ++sp) {
                    int ka, kb;
                    if (dsplits > 0) {
                        ka = static_cast<int>(static_cast<long long>(ctx) * sp / S) / PAGE * PAGE;
                        kb = sp == S - 1 ? ctx : static_cast<int>(static_cast<long long>(ctx) * (sp + 1) / S) / PAGE * PAGE;
                    } else {
                        ka = sp * DSPLIT;
                        kb = (sp + 1) * DSPLIT < ctx ? (sp + 1) * DSPLIT : ctx;
                    }
                    ditems.push_back({t, L0, 0, 1, h, ka, kb, sq, S > 1 ? nparts++ : -1});
                }
            }
            if (S > 1) ctok.push_back(t);
        } else if (n > TC_MIN_ROWS && b->kv16) {
            // long runs of new rows: tensor-core attention, per kv head (both
            // of its query heads in one CTA)
            for (int qa = 0; qa < n; qa += TA_ROWS)
                for (int h = 0; h < HKV; ++h)
                    titems.push_back({t, L0, qa, qa + TA_ROWS < n ? qa + TA_ROWS : n, h, 0, L0 + n, sq, -1});
        } else {
            for (int qa = 0; qa < n; qa += AQB)
                for (int h = 0; h < HKV; ++h)
                    pitems.push_back({t, L0, qa, qa + AQB < n ? qa + AQB : n, h, 0, L0 + n, sq, -1});
        }
        t += n;
    }
    // the longest tensor-core attention items first (their key count sets
    // the work), so that the short ones fill the last wave
    std::stable_sort(titems.begin(), titems.end(),
                     [](const AttnItem &a, const AttnItem &c) { return a.L0 + a.qb > c.L0 + c.qb; });
    if (static_cast<size_t>(nparts) > b->max_parts)
        return set_err(QTTS_E_CAPACITY, "qtts_batch_forward: too many attention splits");
    // tok_seq | tok_pos | prefill items | decode items | cfirst | ccount | ctok | last
    std::vector<int> meta;
    meta.insert(meta.end(), tok_seq.begin(), tok_seq.end());
    meta.insert(meta.end(), tok_pos.begin(), tok_pos.end());
    const int *ip = reinterpret_cast<const int *>(pitems.data());
    meta.insert(meta.end(), ip, ip + pitems.size() * (sizeof(AttnItem) / 4));
    P->o_ditems = meta.size();
    ip = reinterpret_cast<const int *>(ditems.data());
    meta.insert(meta.end(), ip, ip + ditems.size() * (sizeof(AttnItem) / 4));
    P->o_titems = meta.size();
    ip = reinterpret_cast<const int *>(titems.data());
    meta.insert(meta.end(), ip, ip + titems.size() * (sizeof(AttnItem) / 4));
    P->o_cf = meta.size();
    meta.insert(meta.end(), cfirst.begin(), cfirst.end());
    P->o_cc = meta.size();
    meta.insert(meta.end(), ccount.begin(), ccount.end());
    P->o_ct = meta.size();
    meta.insert(meta.end(), ctok.begin(), ctok.end());
    P->o_last = meta.size();
    meta.insert(meta.end(), last.begin(), last.end());
    if (meta.size() * 4 > b->meta_bytes) return set_err(QTTS_E_CAPACITY, "qtts_batch_forward: too many attention items");
    int *hm;
    if (fixed >= 0) {
        if (fixed >= qtts_batch::NFIXED) return set_err(QTTS_E_ARG, "qtts_batch_forward: fixed slot %d", fixed);
        if (!b->hfixed[fixed] && cudaHostAlloc(reinterpret_cast<void **>(&b->hfixed[fixed]),
                                               b->meta_bytes + b->h_pages.size() * 4, cudaHostAllocDefault) != cudaSuccess) {
            b->hfixed[fixed] = nullptr;
            return set_err(QTTS_E_OOM, "qtts_batch_forward: out of pinned host memory");
        }
        hm = b->hfixed[fixed];
        P->ring = -1;
    } else {
        // the next ring slot, once the copy that last used it has run
        const int k = b->mslot;
        b->mslot = (k + 1) % qtts_batch::NSLOT;
        if (b->mev_live[k]) CK(cudaEventSynchronize(b->mev[k]));
        hm = b->hmeta[k];
        P->ring = k;
    }
    std::memcpy(hm, meta.data(), meta.size() * 4);
    std::memcpy(hm + b->meta_bytes / 4, b->h_pages.data(), b->h_pages.size() * 4);
    P->hm = hm;
    P->nseq = nseq;
    P->T = T;
    P->np = static_cast<int>(pitems.size());
    P->nd = static_cast<int>(ditems.size());
    P->ntc = static_cast<int>(titems.size());
    P->ncomb = static_cast<int>(ctok.size());
    P->meta_ints = meta.size();
    for (int i = 0; i < nseq; ++i) b->len[seqs[i]] += rows[i];
    return QTTS_OK;
}

// The device half: the metadata and page table to the device, the input
// rows (host or device pointer), the layers, the final norm of the last row
// of each sequence and the head `head` (< 0: none); logits and normed rows
// stay in b->logits / b->hidden in call order.  Nothing waits: device waits
// that give up set b->err (read by the caller).
static int batch_enqueue(qtts_batch *b, const BatchPlan &P, const float *x, bool x_dev, int head, cudaStream_t st) {
    if (!x) return set_err(QTTS_E_ARG, "qtts_batch_forward: NULL rows");
    if (head >= static_cast<int>(b->heads->mats.size()))
        return set_err(QTTS_E_ARG, "qtts_batch_forward: no head %d", head);
    CK(cudaSetDevice(b->dev->ordinal));
    CK(cudaMemcpyAsync(b->meta, P.hm, P.meta_ints * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(b->d_pages, P.hm + b->meta_bytes / 4, b->h_pages.size() * 4, cudaMemcpyHostToDevice, st));
    if (P.ring >= 0) {
        CK(cudaEventRecord(b->mev[P.ring], st));
        b->mev_live[P.ring] = true;
    }
    CK(cudaMemcpyAsync(b->x, x, static_cast<size_t>(P.T) * H * 4,
                       x_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
    const int wdt = b->stack->cfg.dtype == QTTS_DTYPE_F32 ? WDT_F32 : WDT_Q8;
    int rc = QTTS_OK;
    const int *m = b->meta;
    const AttnItem *d_pitems = reinterpret_cast<const AttnItem *>(m + 2 * P.T);
    const AttnItem *d_ditems = reinterpret_cast<const AttnItem *>(m + P.o_ditems);
    const AttnItem *d_titems = reinterpret_cast<const AttnItem *>(m + P.o_titems);
    if (b->kv_dtype == QTTS_DTYPE_F32)
        batch_layers<float>(b, P.T, P.np, d_pitems, P.nd, d_ditems, P.ntc, d_titems, m, m + P.T, P.ncomb, m + P.o_cf,
                            m + P.o_cc, m + P.o_ct, wdt, st, rc);
    else
        batch_layers<__nv_bfloat16>(b, P.T, P.np, d_pitems, P.nd, d_ditems, P.ntc, d_titems, m, m + P.T, P.ncomb,
                                    m + P.o_cf, m + P.o_cc, m + P.o_ct, wdt, st, rc);
    if (rc) return rc;
    const int hr = head >= 0 ? b->heads->mats[head].rows : 0;
    CK(launch_pdl(rmsnorm_f16_kernel, dim3(norm_grid(P.nseq)), dim3(256), 0, st, static_cast<const float *>(b->x),
                  m + P.o_last, P.nseq, static_cast<const float *>(b->stack->d_final_norm), b->stack->cfg.rms_eps,
                  b->hlast16, b->hidden));
    if (head >= 0) {
        const HeadMat &hm = b->heads->mats[head];
        if ((rc = gemm(hm.t, wdt, hm.rows, H, b->hlast16, P.nseq, b->max_seqs, b->logits, hm.rows, false, b->err, st)))
            return rc;
    }
    return QTTS_OK;
}

// plan + enqueue (the ring of pinned slots, splits by DSPLIT)
static int batch_run(qtts_batch *b, int nseq, const int32_t *seqs, const int32_t *rows, const float *x, bool x_dev,
                     int head, cudaStream_t st) {
    BatchPlan P;
    int rc = batch_plan(b, nseq, seqs, rows, 0, -1, &P);
    if (rc) return rc;
    return batch_enqueue(b, P, x, x_dev, head, st);
}

extern "C" int qtts_batch_forward(qtts_batch *b, int nseq, const int32_t *seqs, const int32_t *rows, const float *x,
                                  int head, float *logits, float *hidden) {
    if (!b) return set_err(QTTS_E_ARG, "qtts_batch_forward: NULL batch");
    if (logits && (head < 0 || head >= static_cast<int>(b->heads->mats.size())))
        return set_err(QTTS_E_ARG, "qtts_batch_forward: no head %d", head);
    CK(cudaSetDevice(b->dev->ordinal));
    cudaStream_t st = b->stream;
    CK(cudaMemsetAsync(b->err, 0, 16, st));
    std::vector<int> saved(b->len);
    int rc = batch_run(b, nseq, seqs, rows, x, false, logits ? head : -1, st);
    if (rc) {
        b->len = saved;
        return rc;
    }
    int err = 0;
    const int hr = logits ? b->heads->mats[head].rows : 0;
    CK(cudaMemcpyAsync(&err, b->err, 4, cudaMemcpyDeviceToHost, st));
    if (logits) CK(cudaMemcpyAsync(logits, b->logits, static_cast<size_t>(nseq) * hr * 4, cudaMemcpyDeviceToHost, st));
    if (hidden) CK(cudaMemcpyAsync(hidden, b->hidden, static_cast<size_t>(nseq) * H * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (err) {
        b->len = saved;
        return set_err(QTTS_E_TIMEOUT, "qtts_batch_forward: a device wait gave up");
    }
    return QTTS_OK;
}

extern "C" int qtts_batch_destroy(qtts_batch *b) {
    if (!b) return QTTS_OK;
    cudaSetDevice(b->dev->ordinal);
    batch_free(b);
    return QTTS_OK;
}

// ------------------------------------------------------------------ batched frames
//
// qtts_talkers: TQwenTalker (greedy) for many utterances at once over a
// talker batch and a predictor batch.  The state of every utterance lives on
// the device; a frame is 15 predictor calls and one talker call over all
// active utterances, queued back to back with the choices between them,
// and one read of the codes at its end.

struct qtts_talkers {
    qtts_batch *tb, *pb;
    qtts_talker_config cfg;
    cudaStream_t stream;
    float *codec_emb, *pred_emb, *tts_pad, *hid, *px, *xt;
    const float **d_trail;
    std::vector<float *> trail;  // per utterance, device (NULL: none)
    SeqState *ss;
    unsigned char *seen;
    int *d_seqs, *d_aux, *d_codes, *d_done;
    int *h_io;  // pinned: seqs | aux | codes | done | errs
    std::vector<char> started, done;
    std::vector<int> last_talker;  // the utterances of the last talker call, in its row order
    std::vector<void *> allocs;
    // the frame as one CUDA graph, for one list of active utterances; its
    // calls read their metadata from fixed pinned slots rewritten each frame
    cudaGraphExec_t graph = nullptr;
    std::vector<int> graph_seqs;
    BatchPlan graph_plans[MAX_GROUPS];
    int frames_eager = 0, frames_graph = 0, captures = 0;
    SampleParams samp0 = {}, samp = {};  // code 0 / the predictor's codes (on = 0: greedy)
    uint64_t seed = 0;                   // utterance s draws from stream seed + s
};

static void talkers_free(qtts_talkers *t) {
    if (t->graph) cudaGraphExecDestroy(t->graph);
    for (float *p : t->trail)
        if (p) cudaFree(p);
    for (void *p : t->allocs) cudaFree(p);
    if (t->h_io) cudaFreeHost(t->h_io);
    delete t;
}

extern "C" int qtts_talkers_create(qtts_batch *talker, qtts_batch *pred, const qtts_talker_config *c,
                                   const float *codec_emb, const float *pred_emb, qtts_talkers **out) {
    if (!talker || !pred || !c || !codec_emb || !pred_emb || !out)
        return set_err(QTTS_E_ARG, "qtts_talkers_create: NULL argument");
    *out = nullptr;
    if (talker->dev != pred->dev) return set_err(QTTS_E_ARG, "qtts_talkers_create: batches on different devices");
    if (c->groups < 2 || c->groups > MAX_GROUPS || c->vocab <= 1024 || c->pred_vocab <= 0 || c->codec_eos < 0 ||
        c->codec_eos >= c->vocab || !(c->repetition_penalty > 0.f))
        return set_err(QTTS_E_ARG, "qtts_talkers_create: bad talker configuration");
    if (talker->heads->mats.size() != 1 || talker->heads->mats[0].rows != c->vocab)
        return set_err(QTTS_E_ARG, "qtts_talkers_create: the talker needs one head of %d rows", c->vocab);
    if (static_cast<int>(pred->heads->mats.size()) != c->groups - 1)
        return set_err(QTTS_E_ARG, "qtts_talkers_create: the predictor needs %d heads", c->groups - 1);
    for (const HeadMat &m : pred->heads->mats)
        if (m.rows != c->pred_vocab) return set_err(QTTS_E_ARG, "qtts_talkers_create: predictor head rows");
    const int S = talker->max_seqs;
    if (pred->max_seqs < S || pred->max_pos < c->groups || pred->max_tokens < 2 * S)
        return set_err(QTTS_E_ARG,
                       "qtts_talkers_create: the predictor batch needs >= %d sequences, %d positions, %d rows", S,
                       c->groups, 2 * S);
    CK(cudaSetDevice(talker->dev->ordinal));
    qtts_talkers *t = new qtts_talkers();
    t->tb = talker;
    t->pb = pred;
    t->cfg = *c;
    t->stream = talker->stream;
    t->trail.assign(S, nullptr);
    t->started.assign(S, 0);
    t->done.assign(S, 0);
    const size_t G = c->groups;
    struct A {
        void **p;
        size_t bytes;
    } want[] = {
        {reinterpret_cast<void **>(&t->codec_emb), static_cast<size_t>(c->vocab) * H * 4},
        {reinterpret_cast<void **>(&t->pred_emb), (G - 1) * c->pred_vocab * H * 4},
        {reinterpret_cast<void **>(&t->tts_pad), static_cast<size_t>(S) * H * 4},
        {reinterpret_cast<void **>(&t->hid), static_cast<size_t>(S) * H * 4},
        {reinterpret_cast<void **>(&t->px), static_cast<size_t>(2 * S) * H * 4},
        {reinterpret_cast<void **>(&t->xt), static_cast<size_t>(S) * H * 4},
        {reinterpret_cast<void **>(&t->d_trail), static_cast<size_t>(S) * sizeof(float *)},
        {reinterpret_cast<void **>(&t->ss), static_cast<size_t>(S) * sizeof(SeqState)},
        {reinterpret_cast<void **>(&t->seen), static_cast<size_t>(S) * c->vocab},
        {reinterpret_cast<void **>(&t->d_seqs), static_cast<size_t>(S) * 4},
        {reinterpret_cast<void **>(&t->d_aux), static_cast<size_t>(S) * 4},
        {reinterpret_cast<void **>(&t->d_codes), static_cast<size_t>(S) * G * 4},
        {reinterpret_cast<void **>(&t->d_done), static_cast<size_t>(S) * 4},
    };
    for (const A &a : want) {
        if (cudaMalloc(a.p, a.bytes) != cudaSuccess) {
            talkers_free(t);
            return set_err(QTTS_E_OOM, "qtts_talkers_create: out of device memory (%zu bytes)", a.bytes);
        }
        t->allocs.push_back(*a.p);
    }
    if (cudaHostAlloc(reinterpret_cast<void **>(&t->h_io), (static_cast<size_t>(S) * (G + 3) + 8) * 4,
                      cudaHostAllocDefault) != cudaSuccess) {
        talkers_free(t);
        return set_err(QTTS_E_OOM, "qtts_talkers_create: out of pinned host memory");
    }
    if (cudaMemcpy(t->codec_emb, codec_emb, static_cast<size_t>(c->vocab) * H * 4, cudaMemcpyHostToDevice) !=
            cudaSuccess ||
        cudaMemcpy(t->pred_emb, pred_emb, (G - 1) * c->pred_vocab * H * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(t->d_trail, 0, static_cast<size_t>(S) * sizeof(float *)) != cudaSuccess) {
        talkers_free(t);
        return set_err(QTTS_E_CUDA, "qtts_talkers_create: upload failed");
    }
    *out = t;
    return QTTS_OK;
}

// the pinned I/O area: [S] seqs | [S] aux | [S*G] codes | [S] done | [8] errs
static int *io_seqs(qtts_talkers *t) { return t->h_io; }
static int *io_aux(qtts_talkers *t) { return t->h_io + t->tb->max_seqs; }
static int *io_codes(qtts_talkers *t) { return t->h_io + 2 * t->tb->max_seqs; }
static int *io_done(qtts_talkers *t) { return t->h_io + (2 + t->cfg.groups) * t->tb->max_seqs; }
static int *io_errs(qtts_talkers *t) { return t->h_io + (3 + t->cfg.groups) * t->tb->max_seqs; }

static int distinct_seqs(const qtts_talkers *t, int nseq, const int32_t *seqs, const char *who) {
    if (nseq <= 0 || nseq > t->tb->max_seqs || !seqs) return set_err(QTTS_E_ARG, "%s: bad sequence list", who);
    std::vector<char> seen(t->tb->max_seqs, 0);
    for (int i = 0; i < nseq; ++i) {
        if (seqs[i] < 0 || seqs[i] >= t->tb->max_seqs || seen[seqs[i]])
            return set_err(QTTS_E_ARG, "%s: entry %d: sequence %d", who, i, seqs[i]);
        seen[seqs[i]] = 1;
    }
    return QTTS_OK;
}

// both batches' error words, read after the stream has drained
static int talkers_finish(qtts_talkers *t, const char *who) {
    cudaStream_t st = t->stream;
    int *e = io_errs(t);
    CK(cudaMemcpyAsync(e, t->tb->err, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(e + 1, t->pb->err, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (e[0] || e[1]) return set_err(QTTS_E_TIMEOUT, "%s: a device wait gave up", who);
    return QTTS_OK;
}

// rows_dev: prefill, trailing and tts_pad are device rows (the prompts built
// on the device, queued on t->stream), else host rows
static int talkers_start(qtts_talkers *t, int nseq, const int32_t *seqs, const int32_t *rows, const float *prefill,
                         const int32_t *trailing_rows, const float *trailing, const float *tts_pad, bool rows_dev) {
    if (!t || !rows || !prefill || !tts_pad) return set_err(QTTS_E_ARG, "qtts_talkers_start: NULL argument");
    const cudaMemcpyKind kind = rows_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    int rc = distinct_seqs(t, nseq, seqs, "qtts_talkers_start");
    if (rc) return rc;
    size_t ntrail = 0;
    for (int i = 0; i < nseq; ++i) {
        const int tr = trailing_rows ? trailing_rows[i] : 0;
        if (rows[i] <= 0 || tr < 0) return set_err(QTTS_E_ARG, "qtts_talkers_start: entry %d: bad row counts", i);
        if (rows[i] > t->tb->max_pos)
            return set_err(QTTS_E_CAPACITY, "qtts_talkers_start: %d prefill rows, at most %d", rows[i], t->tb->max_pos);
        ntrail += tr;
    }
    if (ntrail > 0 && !trailing) return set_err(QTTS_E_ARG, "qtts_talkers_start: NULL trailing rows");
    CK(cudaSetDevice(t->tb->dev->ordinal));
    cudaStream_t st = t->stream;
    CK(cudaStreamSynchronize(st));
    // the utterances' trailing text rows and tts_pad
    const float *src = trailing;
    for (int i = 0; i < nseq; ++i) {
        const int s = seqs[i], tr = trailing_rows ? trailing_rows[i] : 0;
        t->started[s] = 0;
        if (t->trail[s]) cudaFree(t->trail[s]);
        t->trail[s] = nullptr;
        if (tr > 0) {
            if (cudaMalloc(&t->trail[s], static_cast<size_t>(tr) * H * 4) != cudaSuccess)
                return set_err(QTTS_E_OOM, "qtts_talkers_start: out of device memory");
            CK(cudaMemcpy(t->trail[s], src, static_cast<size_t>(tr) * H * 4, kind));
            src += static_cast<size_t>(tr) * H;
        }
        CK(cudaMemcpy(t->d_trail + s, &t->trail[s], sizeof(float *), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(t->tts_pad + static_cast<size_t>(s) * H, tts_pad, H * 4, kind));
        qtts_batch_reset(t->tb, s);
        io_seqs(t)[i] = s;
        io_aux(t)[i] = tr;
    }
    CK(cudaMemcpyAsync(t->d_seqs, io_seqs(t), nseq * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(t->d_aux, io_aux(t), nseq * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemsetAsync(t->tb->err, 0, 16, st));
    CK(cudaMemsetAsync(t->pb->err, 0, 16, st));
    frames_start_kernel<<<nseq, 256, 0, st>>>(t->d_seqs, t->d_aux, t->ss, t->seen, t->cfg.vocab);
    CK(cudaGetLastError());
    if ((rc = batch_run(t->tb, nseq, seqs, rows, prefill, rows_dev, 0, st))) return rc;
    frames_choose0_kernel<<<nseq, 256, 0, st>>>(t->d_seqs, t->tb->logits, t->tb->hidden, t->cfg.vocab,
                                                t->cfg.codec_eos, t->cfg.repetition_penalty, t->seen, t->ss, t->hid,
                                                t->d_done, 1, t->samp0, static_cast<unsigned long long>(t->seed));
    CK(cudaGetLastError());
    if ((rc = talkers_finish(t, "qtts_talkers_start"))) return rc;
    t->last_talker.assign(seqs, seqs + nseq);
    for (int i = 0; i < nseq; ++i) {
        t->started[seqs[i]] = 1;
        t->done[seqs[i]] = 0;  // eos is forbidden before 2 frames
    }
    return QTTS_OK;
}

extern "C" int qtts_talkers_start(qtts_talkers *t, int nseq, const int32_t *seqs, const int32_t *rows,
                                  const float *prefill, const int32_t *trailing_rows, const float *trailing,
                                  const float *tts_pad) {
    return talkers_start(t, nseq, seqs, rows, prefill, trailing_rows, trailing, tts_pad, false);
}

extern "C" int qtts_talkers_start_prompt(qtts_talkers *t, qtts_textproj *tp, const qtts_prompt_tokens *tok, int nseq,
                                         const int32_t *seqs, const int32_t *ids, const int32_t *n_ids,
                                         const int32_t *codec, const int32_t *n_codec, const int32_t *non_streaming) {
    const char *fn = "qtts_talkers_start_prompt";
    if (!t || !tp || !seqs || !ids || !n_ids || !codec || !n_codec || nseq <= 0)
        return set_err(QTTS_E_ARG, "%s: NULL argument or no utterance", fn);
    // every utterance's rows as (text token, codec id): the prefill rows of
    // all utterances in order, then their trailing rows, then tts_pad
    std::vector<int32_t> rows(nseq), trs(nseq), pt, pc, tt, tc;
    size_t io = 0, co = 0;
    for (int i = 0; i < nseq; ++i) {
        if (n_ids[i] < 0 || n_codec[i] < 0) return set_err(QTTS_E_ARG, "%s: entry %d: negative count", fn, i);
        PromptPlan p;
        int rc = prompt_plan(fn, t->tb->dev, t->cfg.vocab, tp, tok, ids + io, n_ids[i], codec + co, n_codec[i],
                             non_streaming ? non_streaming[i] : 0, p);
        if (rc) return rc;
        rows[i] = p.rows;
        trs[i] = p.trailing;
        pt.insert(pt.end(), p.text.begin(), p.text.begin() + p.rows);
        pc.insert(pc.end(), p.codec.begin(), p.codec.begin() + p.rows);
        tt.insert(tt.end(), p.text.begin() + p.rows, p.text.begin() + p.rows + p.trailing);
        tc.insert(tc.end(), p.codec.begin() + p.rows, p.codec.begin() + p.rows + p.trailing);
        io += static_cast<size_t>(n_ids[i]);
        co += static_cast<size_t>(n_codec[i]);
    }
    const size_t R = pt.size(), T = tt.size();
    pt.insert(pt.end(), tt.begin(), tt.end());
    pc.insert(pc.end(), tc.begin(), tc.end());
    pt.push_back(tok->tts_pad);
    pc.push_back(-1);
    int rc = textproj_run(tp, pt.data(), pc.data(), t->codec_emb, static_cast<int>(pt.size()), t->stream);
    if (rc) return rc;
    const float *y = tp->y;
    return talkers_start(t, nseq, seqs, rows.data(), y, trs.data(), y + R * H, y + (R + T) * H, true);
}

// context splits per sequence of the batched talker step: about 4 waves of
// the decode attention CTAs (6 resident per SM with a bf16 cache) over all
// (utterance, kv head) pairs, 2 to DMAX_SPLITS
static int talker_splits(const qtts_talkers *t, int n) {
    const int want = (24 * t->tb->dev->sms + n * HKV / 2) / (n * HKV);
    return want < 2 ? 2 : (want > DMAX_SPLITS ? DMAX_SPLITS : want);
}

// the device work of one frame of n utterances (plans[0..G-2]: predictor
// steps, plans[G-1]: talker step), queued on st (or captured)
static int frame_enqueue(qtts_talkers *t, int n, const BatchPlan *plans, cudaStream_t st) {
    const int G = t->cfg.groups, pv = t->cfg.pred_vocab;
    int rc;
    CK(cudaMemcpyAsync(t->d_seqs, io_seqs(t), n * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemsetAsync(t->tb->err, 0, 16, st));
    CK(cudaMemsetAsync(t->pb->err, 0, 16, st));
    CK(launch_pdl(frames_begin_kernel, dim3(n), dim3(256), 0, st, static_cast<const int *>(t->d_seqs), t->ss, t->seen,
                  t->cfg.vocab, static_cast<const float *>(t->hid), static_cast<const float *>(t->codec_emb), t->px,
                  t->d_codes, G));
    for (int g = 0; g < G - 1; ++g) {
        if ((rc = batch_enqueue(t->pb, plans[g], t->px, true, g, st))) return rc;
        CK(launch_pdl(frames_pred_argmax_kernel, dim3(n), dim3(256), 0, st, static_cast<const float *>(t->pb->logits),
                      pv, g, G, static_cast<const float *>(t->pred_emb), t->px, t->d_codes,
                      static_cast<const int *>(t->d_seqs), static_cast<const SeqState *>(t->ss), t->samp,
                      static_cast<unsigned long long>(t->seed)));
    }
    CK(launch_pdl(frames_talker_in_kernel, dim3(n), dim3(256), 0, st, static_cast<const int *>(t->d_seqs),
                  static_cast<const SeqState *>(t->ss), static_cast<const int *>(t->d_codes), G,
                  static_cast<const float *>(t->codec_emb), static_cast<const float *>(t->pred_emb), pv,
                  static_cast<const float *const *>(t->d_trail), static_cast<const float *>(t->tts_pad), t->xt));
    if ((rc = batch_enqueue(t->tb, plans[G - 1], t->xt, true, 0, st))) return rc;
    CK(launch_pdl(frames_choose0_kernel, dim3(n), dim3(256), 0, st, static_cast<const int *>(t->d_seqs),
                  static_cast<const float *>(t->tb->logits), static_cast<const float *>(t->tb->hidden), t->cfg.vocab,
                  t->cfg.codec_eos, t->cfg.repetition_penalty, static_cast<const unsigned char *>(t->seen), t->ss,
                  t->hid, t->d_done, 0, t->samp0, static_cast<unsigned long long>(t->seed)));
    CK(cudaMemcpyAsync(io_codes(t), t->d_codes, static_cast<size_t>(n) * G * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(io_done(t), t->d_done, n * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(io_errs(t), t->tb->err, 4, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(io_errs(t) + 1, t->pb->err, 4, cudaMemcpyDeviceToHost, st));
    return QTTS_OK;
}

extern "C" int qtts_talkers_next_frame(qtts_talkers *t, int nseq, const int32_t *seqs, int32_t *codes,
                                       int32_t *more) {
    if (!t || !codes || !more) return set_err(QTTS_E_ARG, "qtts_talkers_next_frame: NULL argument");
    int rc = distinct_seqs(t, nseq, seqs, "qtts_talkers_next_frame");
    if (rc) return rc;
    const int G = t->cfg.groups;
    std::vector<int> act, slot;
    for (int i = 0; i < nseq; ++i) {
        const int s = seqs[i];
        if (!t->started[s]) return set_err(QTTS_E_STATE, "qtts_talkers_next_frame: sequence %d not started", s);
        more[i] = 0;
        if (t->done[s]) continue;
        if (t->tb->len[s] + 1 > t->tb->max_pos)
            return set_err(QTTS_E_CAPACITY, "qtts_talkers_next_frame: sequence %d: talker cache full (%d positions)",
                           s, t->tb->max_pos);
        act.push_back(s);
        slot.push_back(i);
    }
    const int n = static_cast<int>(act.size());
    if (n == 0) return QTTS_OK;
    CK(cudaSetDevice(t->tb->dev->ordinal));
    cudaStream_t st = t->stream;
    // host half of every call of the frame: predictor Reset, [state,
    // codec_emb[code 0]] with head 0, then one row per group with head g
    // (talker.pas:656-675); the talker step
    const std::vector<int> tlen(t->tb->len);
    BatchPlan plans[MAX_GROUPS];
    for (int s : act) qtts_batch_reset(t->pb, s);
    std::vector<int> rows(n, 2);
    for (int g = 0; g < G - 1 && rc == QTTS_OK; ++g) {
        rc = batch_plan(t->pb, n, act.data(), rows.data(), 1, g, &plans[g]);
        if (g == 0) rows.assign(n, 1);
    }
    if (rc == QTTS_OK) rc = batch_plan(t->tb, n, act.data(), rows.data(), talker_splits(t, n), 0, &plans[G - 1]);
    if (rc) {
        t->tb->len = tlen;
        return rc;
    }
    std::memcpy(io_seqs(t), act.data(), n * 4);
    bool reuse = t->graph && t->graph_seqs == act;
    for (int g = 0; g < G && reuse; ++g) reuse = plans[g].same_shape(t->graph_plans[g]);
    if (!reuse) {
        if (t->graph) CK(cudaGraphExecDestroy(t->graph));
        t->graph = nullptr;
        cudaGraph_t g = nullptr;
        CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        rc = frame_enqueue(t, n, plans, st);
        const cudaError_t ce = cudaStreamEndCapture(st, &g);
        if (rc == QTTS_OK && ce != cudaSuccess) rc = set_err(QTTS_E_CUDA, "frame graph capture: %s", cudaGetErrorString(ce));
        if (rc == QTTS_OK && cudaGraphInstantiate(&t->graph, g, 0) != cudaSuccess) {
            t->graph = nullptr;
            rc = set_err(QTTS_E_CUDA, "frame graph: instantiation failed");
        }
        if (g) cudaGraphDestroy(g);
        if (rc) {
            t->tb->len = tlen;
            return rc;
        }
        t->graph_seqs = act;
        for (int k = 0; k < G; ++k) t->graph_plans[k] = plans[k];
        ++t->captures;
    }
    CK(cudaGraphLaunch(t->graph, st));
    CK(cudaStreamSynchronize(st));
    ++t->frames_graph;
    t->last_talker = act;
    if (io_errs(t)[0] || io_errs(t)[1]) return set_err(QTTS_E_TIMEOUT, "qtts_talkers_next_frame: a device wait gave up");
    for (int j = 0; j < n; ++j) {
        std::memcpy(codes + static_cast<size_t>(slot[j]) * G, io_codes(t) + static_cast<size_t>(j) * G, G * 4);
        more[slot[j]] = 1;
        t->done[act[j]] = io_done(t)[j] ? 1 : 0;
    }
    return QTTS_OK;
}

extern "C" int qtts_talkers_probe(qtts_talkers *t, int seq, float *logits, float *hidden) {
    if (!t) return set_err(QTTS_E_ARG, "qtts_talkers_probe: NULL talkers");
    if (seq < 0 || seq >= t->tb->max_seqs) return set_err(QTTS_E_ARG, "qtts_talkers_probe: bad sequence %d", seq);
    int row = -1;
    for (size_t i = 0; i < t->last_talker.size(); ++i)
        if (t->last_talker[i] == seq) row = static_cast<int>(i);
    if (row < 0) return set_err(QTTS_E_STATE, "qtts_talkers_probe: sequence %d took no part in the last talker call", seq);
    CK(cudaSetDevice(t->tb->dev->ordinal));
    CK(cudaStreamSynchronize(t->stream));
    if (logits)
        CK(cudaMemcpy(logits, t->tb->logits + static_cast<size_t>(row) * t->cfg.vocab, static_cast<size_t>(t->cfg.vocab) * 4,
                      cudaMemcpyDeviceToHost));
    if (hidden) CK(cudaMemcpy(hidden, t->hid + static_cast<size_t>(seq) * H, H * 4, cudaMemcpyDeviceToHost));
    return QTTS_OK;
}

extern "C" int qtts_talkers_stream(qtts_talkers *t, void **stream) {
    if (!t || !stream) return set_err(QTTS_E_ARG, "qtts_talkers_stream: NULL argument");
    *stream = t->stream;
    return QTTS_OK;
}

extern "C" int qtts_talkers_destroy(qtts_talkers *t) {
    if (!t) return QTTS_OK;
    cudaSetDevice(t->tb->dev->ordinal);
    cudaStreamSynchronize(t->stream);
    talkers_free(t);
    return QTTS_OK;
}

extern "C" int qtts_talkers_set_sampling(qtts_talkers *t, const qtts_sampling *s) {
    if (!t || !s) return set_err(QTTS_E_ARG, "qtts_talkers_set_sampling: NULL argument");
    SampleParams a, b;
    int rc = sampling_params("qtts_talkers_set_sampling", s->do_sample, s->temperature, s->top_k, s->top_p, &a);
    if (rc) return rc;
    rc = sampling_params("qtts_talkers_set_sampling (predictor)", s->sub_do_sample, s->sub_temperature, s->sub_top_k,
                         s->sub_top_p, &b);
    if (rc) return rc;
    if (t->cfg.vocab > SAMPLE_MAX_V || t->cfg.pred_vocab > SAMPLE_MAX_V)
        return set_err(QTTS_E_ARG, "qtts_talkers_set_sampling: vocabularies of %d / %d, at most %d", t->cfg.vocab,
                       t->cfg.pred_vocab, SAMPLE_MAX_V);
    CK(cudaSetDevice(t->tb->dev->ordinal));
    CK(cudaStreamSynchronize(t->stream));
    t->samp0 = a;
    t->samp = b;
    t->seed = s->seed;
    // the captured frame holds the old options
    if (t->graph) {
        cudaGraphExecDestroy(t->graph);
        t->graph = nullptr;
        t->graph_seqs.clear();
    }
    return QTTS_OK;
}

// ------------------------------------------------------------------ the 12 Hz codec

#include "qtts_codec.cuh"
