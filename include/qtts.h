/*
 * qtts.h -- C-ABI of libqtts.so, the B200 (sm_100a) implementation of the
 * per-frame language-model path of mormot2-qwen-tts: the Qwen3-TTS talker
 * (28 layers, code 0 of each 80 ms frame) and the 5-layer code predictor
 * (codes 1..15), with their heads.
 *
 * The library sits UNDER the reference's Object Pascal stack API
 * (src/tts/mormot.ai.tts.qwen.lm.pas, mormot.ai.tts.qwen.talker.pas).  Each
 * entry point below names the reference call it replaces (file:line in the
 * reference project).  Plain C types only: pointers, sizes, ints.
 *
 * Conventions
 *  - Every entry returns an int: QTTS_OK (0) or a QTTS_E_* code.  Nothing
 *    aborts the process.  qtts_last_error() gives the message of the last
 *    failure of the calling thread (the Pascal side raises EQwenLm with it,
 *    as lm.pas:167, 232-234 and 345 raise on bad shapes).
 *  - Host pointers given to a create/add call are copied to the device
 *    during the call; the caller may free them afterwards.  Weights are never
 *    keyed by host address (the stale-weights issue of the reference's
 *    README "Device weights are keyed by their host address" cannot occur).
 *  - Ownership: qtts_lm_create takes ownership of its stack (as
 *    TQwenLm.Create owns its TDecoderModel, lm.pas:118-123) but not of its
 *    heads, which must outlive it.  Destroy order: talker, lm, heads, device.
 *  - Threading: one lm or talker per thread, as TQwenTalker is "not to be
 *    shared between threads" (talker.pas:77).  One device may serve several.
 *  - Model dimensions: hidden 1024, 16 query heads, 8 KV heads, head_dim
 *    128, intermediate 3072 (the two stacks of Qwen3-TTS-12Hz-0.6B); other
 *    dimensions are rejected with QTTS_E_ARG.  Layers and head rows are free.
 */
#ifndef QTTS_H
#define QTTS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QTTS_OK 0
#define QTTS_E_ARG 1      /* bad argument, shape or handle */
#define QTTS_E_OOM 2      /* device memory exhausted */
#define QTTS_E_CUDA 3     /* a CUDA call failed */
#define QTTS_E_CAPACITY 4 /* the KV cache is full (position >= max_pos) */
#define QTTS_E_TIMEOUT 5  /* a bounded device-side wait gave up */
#define QTTS_E_STATE 6    /* call out of order (e.g. next_frame before start) */

/* weight formats (TInferDType idtF32 / idtQ8_0 / the BF16 of the file) */
#define QTTS_DTYPE_F32 0
#define QTTS_DTYPE_Q8_0 1 /* ggml block_q8_0: fp16 scale + 32 int8, 34 bytes */
#define QTTS_DTYPE_BF16 2 /* source rows only: widened exactly to float32 */
#define QTTS_DTYPE_F16 3  /* a safetensors F16 tensor, or a half-float KV cache (not a weight source) */
#define QTTS_DTYPE_OTHER -1 /* a safetensors tensor of another dtype */
#define QTTS_MAX_DIMS 8   /* dimensions of a safetensors tensor */

typedef struct qtts_device qtts_device;
typedef struct qtts_stack qtts_stack;
typedef struct qtts_heads qtts_heads;
typedef struct qtts_lm qtts_lm;
typedef struct qtts_talker qtts_talker;
typedef struct qtts_textproj qtts_textproj;
typedef struct qtts_safetensors qtts_safetensors;
typedef struct qtts_codec qtts_codec;

/* The decoder configuration of one stack (TDecoderConfig: talker_config or
 * talker_config.code_predictor_config of config.json, talker.pas:252-273).
 * dtype: the format the weights take on the device, F32 or Q8_0. */
typedef struct qtts_stack_config {
    int32_t layers;
    int32_t hidden;
    int32_t heads;
    int32_t kv_heads;
    int32_t head_dim;
    int32_t intermediate;
    float rms_eps;
    float rope_theta;
    int32_t dtype;
} qtts_stack_config;

/* The tensors of one layer, as host pointers.  Matrices are [out][in]
 * (PyTorch nn.Linear layout) in `dtype` (F32 or BF16 rows, or Q8_0 ggml
 * blocks along `in`); norm weights are float32. */
typedef struct qtts_layer_src {
    int32_t dtype;
    const void *q_proj;    /* [heads*head_dim][hidden]     */
    const void *k_proj;    /* [kv_heads*head_dim][hidden]  */
    const void *v_proj;    /* [kv_heads*head_dim][hidden]  */
    const void *o_proj;    /* [hidden][heads*head_dim]     */
    const void *gate_proj; /* [intermediate][hidden]       */
    const void *up_proj;   /* [intermediate][hidden]       */
    const void *down_proj; /* [hidden][intermediate]       */
    const float *input_norm; /* [hidden]   input_layernorm          */
    const float *post_norm;  /* [hidden]   post_attention_layernorm */
    const float *q_norm;     /* [head_dim] */
    const float *k_norm;     /* [head_dim] */
} qtts_layer_src;

/* ------------------------------------------------------------------ device */

/* Opens CUDA device `ordinal` (TQwenVulkan.Create, lm.pas:207-211). */
int qtts_device_open(int ordinal, qtts_device **out);
/* TQwenVulkan.DeviceName (lm.pas:219-222). */
int qtts_device_name(qtts_device *dev, char *buf, int len);
/* TQwenVulkan.DeviceBytes (lm.pas:59-61): bytes of the stack weights held. */
int qtts_device_bytes(qtts_device *dev, int64_t *bytes);
/* TQwenVulkan.Destroy (lm.pas:213-217). */
int qtts_device_close(qtts_device *dev);

/* ------------------------------------------------------------------ stack */

/* One Qwen3 stack on the device: QwenLmStack -> TQwen3Model.CreateStack
 * (lm.pas:174-179) plus the upload of TQwenLm.Create (lm.pas:347-356).
 * layers: config->layers entries; final_norm: [hidden] float32.  F32 or
 * BF16 sources with a Q8_0 config are quantised on the device with ggml's
 * quantize_row_q8_0_ref rule. */
int qtts_stack_create(qtts_device *dev, const qtts_stack_config *config, const qtts_layer_src *layers,
                      const float *final_norm, qtts_stack **out);
/* StackBytes (lm.pas:181-197): bytes of the matrices and norms. */
int qtts_stack_bytes(const qtts_stack *stack, int64_t *bytes);
int qtts_stack_destroy(qtts_stack *stack);

/* ------------------------------------------------------------------ heads */

/* TQwenLmHeads.Create (lm.pas:227-238): dtype F32 or Q8_0, hidden % 32 == 0. */
int qtts_heads_create(qtts_device *dev, const char *name, int hidden, int dtype, qtts_heads **out);
/* TQwenLmHeads.Add (lm.pas:277-308): a [rows][hidden] head from F32 or BF16
 * host rows; *index receives its index.  Q8_0 conversion runs on the device
 * and gives the bytes of ggml's quantize_row_q8_0_ref. */
int qtts_heads_add(qtts_heads *heads, const void *src, int src_dtype, int rows, int *index);
/* TQwenLmHeads.Digest (lm.pas:310-317): crc32c of the stored bytes (ggml
 * blocks for Q8_0, float32 rows otherwise) in load order. */
int qtts_heads_digest(qtts_heads *heads, uint32_t *crc);
/* TQwenLmHeads.Count / Rows / Bytes (lm.pas:88-99). */
int qtts_heads_count(qtts_heads *heads, int *count);
int qtts_heads_rows(qtts_heads *heads, int index, int *rows);
int qtts_heads_bytes(qtts_heads *heads, int64_t *bytes);
/* TInferBackend.Linear on a head (lm.pas:404-406: the reference applies the
 * heads with fCpu.Linear), for many rows at once: y[rows][head rows] =
 * x[rows][hidden] . head^T, host buffers.  Runs the tcgen05 GEMM (fp16
 * operands, f32 accumulation). */
int qtts_heads_linear(qtts_heads *heads, int index, const float *x, int rows, float *y);
int qtts_heads_destroy(qtts_heads *heads);

/* ------------------------------------------------------------------ lm */

/* TQwenLm.Create (lm.pas:337-360): takes ownership of `stack`; `heads` is not
 * owned.  max_pos: KV cache capacity in positions (float32 cache, the
 * reference's default, talker.pas:188-190). */
int qtts_lm_create(qtts_stack *stack, qtts_heads *heads, int max_pos, qtts_lm **out);
/* TQwenLm.Create with its aKvF16 argument (lm.pas:122-123, applied to the
 * device context at lm.pas:352; TQwenTalkerOptions.KvF16, talker.pas:56):
 * kv_dtype QTTS_DTYPE_F32 (as qtts_lm_create) or QTTS_DTYPE_F16, the K/V
 * cache in half floats (round to nearest even; the current position is read
 * back rounded too), half the cache memory and traffic. */
int qtts_lm_create_kv(qtts_stack *stack, qtts_heads *heads, int max_pos, int kv_dtype, qtts_lm **out);
/* TQwenLm.Reset (lm.pas:374-378): the next row is at position 0. */
int qtts_lm_reset(qtts_lm *lm);
/* TQwenLm.Forward (lm.pas:391-408): appends rows x[rows][hidden] at
 * positions Length..Length+rows-1; for the last row, the normed state goes
 * to hidden (may be NULL) and the logits of head `head` to logits (NULL:
 * no head).  rows <= 0 does nothing. */
int qtts_lm_forward(qtts_lm *lm, const float *x, int rows, int head, float *logits, float *hidden);
/* The forward of qtts_lm_forward for callers that must not allocate device
 * memory while they run it: a real-time synthesis thread, for which
 * cudaMalloc/cudaFree (they can synchronise the whole device and block for
 * milliseconds) are off limits, or a host whose GPU memory is all handed out
 * by its own pool allocator.  No counterpart in the reference.  x
 * [rows][hidden], logits (head rows) and hidden [hidden] are DEVICE pointers
 * owned by the caller (logits/hidden may be NULL), each 16-byte aligned
 * (QTTS_E_ARG otherwise, before anything runs); x is read in place.  The
 * call allocates nothing: the kernel's scratch is one static device array of
 * 931,584 bytes (every GPU that loads the library holds it until exit),
 * sized for at most 160 SMs and heads of at most 4096 rows; larger requests
 * fail with QTTS_E_CAPACITY.  qtts_lm_create looks up the array's device
 * address (cudaGetSymbolAddress, which may load the library's module on that
 * device) with its device current, so these calls load nothing; only if that
 * lookup failed does the first call repeat it: then make that first call
 * before any stream capture and outside the real-time thread.  All calls on one GPU
 * share its copy of the array, which keeps the last call's contents (each
 * call first clears the barrier and error words it needs at zero): calls
 * that overlap on the same GPU, from two threads or two lms, race and must
 * be serialised by the caller.  Runs on the lm's stream and returns once the
 * results are in the caller's buffers. */
int qtts_lm_forward_noalloc(qtts_lm *lm, const float *x, int rows, int head, float *logits, float *hidden);
/* TQwenLm.Length (lm.pas:136-138). */
int qtts_lm_length(qtts_lm *lm, int *length);
/* The failure path of the bounded device waits, for tests (the reference
 * bounds its waits and aborts cleanly, mormot.ai.tts.qwen.pas:541-548): the
 * following launches of this lm (forwards, and frames when it is a talker's
 * talker lm) run their grid barriers expecting extra_arrivals (0 or 1) more
 * CTAs than the grid holds -- an arrival that never comes -- with every grid
 * barrier and tagged-word spin bounded by wait_cycles SM clock cycles (0: the
 * default bound, about 2 s).  Such a launch returns QTTS_E_TIMEOUT with the
 * place it gave up; its positions are not appended and the next launch
 * starts clean.  (0, 0) restores normal operation. */
int qtts_lm_set_wait_test(qtts_lm *lm, int extra_arrivals, int64_t wait_cycles);
/* Test knob of the batch-1 kernel's tagged handoffs (no counterpart in the
 * reference).  Values
 * pass between the kernel's CTAs as words tagged with the launch's epoch, a
 * counter of this lm's scratch that wraps after 2^22 - 1 launches, the host
 * clearing the tagged words before epoch 1 comes round again.  This sets
 * the counter (0 .. 2^22 - 1; the next launch of this lm, or of frames when
 * it is a talker's talker lm, uses epoch + 1, or wraps), so that a test can
 * cross the wrap in a few launches. */
int qtts_lm_set_launch_epoch(qtts_lm *lm, uint32_t epoch);
/* TQwenLm.Destroy (lm.pas:362-372): frees the cache, then the stack. */
int qtts_lm_destroy(qtts_lm *lm);

/* ------------------------------------------------------------------ batch */

typedef struct qtts_batch qtts_batch;

/* Many sequences (utterances) through one stack per call: the TQwenLm.Forward
 * protocol (lm.pas:391-408) for a batch, as the batched decode and the
 * batched prefill of the TTS engine need it; no counterpart object in the
 * reference, which runs one TQwenLm per stack.  The stack and the heads are
 * not owned (destroy the batch first).  Up to max_seqs sequences (ids
 * 0..max_seqs-1) of up to max_pos positions, up to max_tokens rows per call;
 * the KV cache is paged (16 positions per page), kv_dtype F32 or BF16.  The
 * projections run on the tcgen05 GEMM (fp16 operands, f32 accumulation). */
int qtts_batch_create(qtts_stack *stack, qtts_heads *heads, int max_seqs, int max_tokens, int max_pos, int kv_dtype,
                      qtts_batch **out);
/* TQwenLm.Reset of one sequence: its pages return to the pool. */
int qtts_batch_reset(qtts_batch *batch, int seq);
/* TQwenLm.Length of one sequence. */
int qtts_batch_length(qtts_batch *batch, int seq, int *length);
/* One call: sequence seqs[i] (distinct) receives rows[i] rows, the rows of
 * all sequences concatenated in x [sum rows][hidden]; for each sequence the
 * normed state of its last row goes to hidden [nseq][hidden] and the logits
 * of head `head` to logits [nseq][head rows] (either may be NULL). */
int qtts_batch_forward(qtts_batch *batch, int nseq, const int32_t *seqs, const int32_t *rows, const float *x, int head,
                       float *logits, float *hidden);
int qtts_batch_destroy(qtts_batch *batch);

/* ------------------------------------------------------------------ talker */

/* The choice of codes and the frame layout of TQwenTalker (talker.pas:
 * 86-111, 193-201): vocab 3072 (talker), pred_vocab 2048, groups 16,
 * codec_eos_token_id, repetition_penalty (1.05 in greedy mode). */
typedef struct qtts_talker_config {
    int32_t vocab;
    int32_t pred_vocab;
    int32_t groups;
    int32_t codec_eos;
    float repetition_penalty;
} qtts_talker_config;

/* The per-frame loop of TQwenTalker on the device (greedy): talker and
 * predictor lms (not owned; their heads: 1 talker head [vocab][hidden], 15
 * predictor heads [pred_vocab][hidden]), the code embeddings of the talker
 * codec_emb [vocab][hidden] and of the predictor pred_emb
 * [groups-1][pred_vocab][hidden], float32 (talker.pas:307-311). */
int qtts_talker_create(qtts_lm *talker, qtts_lm *predictor, const qtts_talker_config *config,
                       const float *codec_emb, const float *pred_emb, qtts_talker **out);
/* The end of TQwenTalker.Start (talker.pas:561-592): the trailing text rows
 * (trailing [trailing_rows][hidden]; tts_pad [hidden] after them), talker
 * Reset + Forward of the prefill rows [rows][hidden], empty history.  The
 * logits of the last row (head 0) and its normed state are returned when
 * the pointers are not NULL. */
int qtts_talker_start(qtts_talker *t, const float *prefill, int rows, const float *trailing, int trailing_rows,
                      const float *tts_pad, float *logits, float *hidden);
/* TQwenTalker.NextFrame (talker.pas:640-681), greedy: ChooseCode0, the
 * predictor (2 rows then 14 steps, each with its head and argmax), the sum
 * of the 16 embeddings plus the trailing row, the talker step.  codes[groups]
 * receives the frame; *more = 0 at eos (codes untouched), 1 otherwise. */
int qtts_talker_next_frame(qtts_talker *t, int32_t *codes, int *more);
/* Up to `frames` NextFrame calls launched back to back with no host round
 * trip between them (the producer loop of TQwenTtsProducer.Execute,
 * mormot.ai.tts.qwen.pas:276-319, without its per-frame hand-over):
 * codes[frames][groups] receives the frames, *produced their count (fewer
 * than `frames` when eos was chosen). */
int qtts_talker_run(qtts_talker *t, int frames, int32_t *codes, int *produced);
/* NextFrame with a phase trace (profiling, the role of the reference's
 * TPrecisionTimer stats, mormot.ai.tts.qwen.pas:86-96): stamps[cap] receives
 * the timestamps of CTA 0 at each phase boundary, (tag << 48) | ns, and *n
 * their count. */
int qtts_talker_trace_frame(qtts_talker *t, int32_t *codes, int *more, uint64_t *stamps, int cap, int *n);
/* The CUDA stream (cudaStream_t) the talker's kernels run on, for callers
 * that time them with events. */
int qtts_talker_stream(qtts_talker *t, void **stream);
/* The talker probes of TQwenTalker.Emit (talker.pas:590, 678): the logits
 * (head 0, [vocab]) and the normed state ([hidden]) of the last talker
 * forward.  Either pointer may be NULL. */
int qtts_talker_probe(qtts_talker *t, float *logits, float *hidden);
/* TQwenTalker.Step (talker.pas:152-154): frames returned since start. */
int qtts_talker_step(qtts_talker *t, int *step);
int qtts_talker_destroy(qtts_talker *t);

/* How each code is chosen: TQwenSampling (talker.pas:60-73), as read by
 * QwenSamplingFromConfig (talker.pas:203-230; qwen_tts defaults: sampling
 * on, temperature 0.9, top_k 50, top_p 1 for both the talker's code 0 and
 * the predictor's codes).  do_sample = 0: greedy (the first maximum).  The
 * draw replaces TInferSampler (mormot2-ai, NewSampler talker.pas:455-469):
 * z = logit / temperature, the values >= the top_k-th largest, the nucleus
 * of mass top_p in (z desc, index asc) order, an inverse-CDF draw whose
 * uniform is a function of (seed, frame, code group) alone (frame = the
 * index of the frame the code belongs to, group = 0 for code 0, g for the
 * predictor's code g).  Limits: temperature > 0, 1 <= top_k <= 64,
 * 0 < top_p <= 1. */
typedef struct qtts_sampling {
    int32_t do_sample;
    float temperature;
    int32_t top_k;
    float top_p;
    int32_t sub_do_sample;
    float sub_temperature;
    int32_t sub_top_k;
    float sub_top_p;
    uint64_t seed;
} qtts_sampling;

/* The sampling of TQwenTalker (its fSampler / fSubSampler, talker.pas:
 * 583-586) for the frames that follow; the draw of the first code 0 is made
 * by qtts_talker_start, so set it before.  A new talker is greedy. */
int qtts_talker_set_sampling(qtts_talker *t, const qtts_sampling *s);
/* TInferSampler.Next (the draw of talker.pas:626-629, 632-638) on the
 * device: the index drawn from work[n] (host float32 logits after the
 * processors, n <= 4096) with draw (step, group) of the stream `seed`.
 * Blocking; it uses a buffer of the device object, so calls on one device
 * from several threads must not overlap. */
int qtts_sample(qtts_device *dev, const float *work, int n, float temperature, int top_k, float top_p,
                uint64_t seed, int step, int group, int32_t *code);

/* ------------------------------------------------------------------ text projection */

/* TQwenTalker.TextProject (talker.pas:390-421), Qwen3TTSTalkerResizeMLP:
 * y = fc2(silu(fc1(text_embedding[id]))) in float32 with biases, for the
 * text rows of the prompt and of the trailing text (talker.pas:532-574).
 * emb [vocab][text_hidden] in emb_dtype (QTTS_DTYPE_BF16 as in the
 * checkpoint, or F32; kept on the device as given), fc1_w
 * [text_hidden][text_hidden], fc1_b [text_hidden], fc2_w
 * [hidden][text_hidden], fc2_b [hidden]; copied at create. */
int qtts_textproj_create(qtts_device *dev, int vocab, int text_hidden, int hidden, int emb_dtype, const void *emb,
                         const float *fc1_w, const float *fc1_b, const float *fc2_w, const float *fc2_b,
                         qtts_textproj **out);
/* y[n][hidden] (host) = the projection of the text tokens ids[n] (host); an
 * id outside [0, vocab) is QTTS_E_ARG, as TextProject raises. */
int qtts_text_project(qtts_textproj *t, const int32_t *ids, int n, float *y);
int qtts_textproj_destroy(qtts_textproj *t);

/* The token ids that TQwenTalker.Start places around the text (config.json,
 * read at talker.pas:256-265): text tokens tts_bos/tts_eos/tts_pad
 * (tts_*_token_id; their rows are projections, talker.pas:339-344) and codec
 * ids codec_pad/codec_bos (talker_config.codec_*_id). */
typedef struct qtts_prompt_tokens {
    int32_t tts_bos;
    int32_t tts_eos;
    int32_t tts_pad;
    int32_t codec_pad;
    int32_t codec_bos;
} qtts_prompt_tokens;

/* The rows of TQwenTalker.Start (talker.pas:528-574) as a plan, on the host
 * (no device): row r of the prefill, then of the trailing text, is the text
 * projection of text_out[r] plus, when codec_out[r] >= 0, the codec
 * embedding of codec_out[r]; *rows / *trailing_rows receive the counts.
 * With text_out and codec_out both NULL only the counts; else they hold cap
 * >= rows + trailing_rows entries.  Arguments as qtts_talker_start_prompt;
 * the ids are not range-checked here (the start does it). */
int qtts_prompt_plan(const qtts_prompt_tokens *tok, const int32_t *ids, int n_ids, const int32_t *codec, int n_codec,
                     int non_streaming, int32_t *text_out, int32_t *codec_out, int cap, int *rows,
                     int *trailing_rows);
/* TQwenTalker.Start (talker.pas:528-592) from token ids, its rows built on
 * the device: ids[n_ids] = PromptIds(text), i.e. [im_start, assistant, \n]
 * text [im_end, \n, im_start, assistant, \n] (n_ids >= 9, as Start's "empty
 * text" check); codec[n_codec] = the think / language / voice ids then
 * codec_pad, codec_bos (talker.pas:515-527; n_codec >= 2); non_streaming =
 * aNonStreaming.  Every prefill and trailing row is the text projection of
 * one token (role, text, tts_pad/bos/eos) plus, for the rows over the
 * codec, the talker's codec embedding of one id (AddRow); then as
 * qtts_talker_start.  A text token outside [0, vocab) or a codec id outside
 * [0, talker vocab) is QTTS_E_ARG.  tp and t on the same device; tp's hidden
 * is the talker's. */
int qtts_talker_start_prompt(qtts_talker *t, qtts_textproj *tp, const qtts_prompt_tokens *tok, const int32_t *ids,
                             int n_ids, const int32_t *codec, int n_codec, int non_streaming, float *logits,
                             float *hidden);
/* The rows qtts_talker_start_prompt builds, copied to the host (the probes
 * talker.prefill.embeds and talker.trailing of Start, talker.pas:575-576):
 * *rows and *trailing_rows receive the counts; with prefill and trailing
 * both NULL only the counts, else prefill [prefill_cap][hidden] and
 * trailing [trailing_cap][hidden] must hold them. */
int qtts_talker_prompt_rows(qtts_talker *t, qtts_textproj *tp, const qtts_prompt_tokens *tok, const int32_t *ids,
                            int n_ids, const int32_t *codec, int n_codec, int non_streaming, float *prefill,
                            int prefill_cap, float *trailing, int trailing_cap, int *rows, int *trailing_rows);

/* ------------------------------------------------------------------ files */

/* TSafeTensorsFile.Create (mormot2-ai; used at talker.pas:299): maps a
 * .safetensors file read-only and reads its header.  A header that is not
 * the format (size, JSON, unknown dtype, data_offsets outside the data or
 * not shape x dtype bytes, a name twice) is QTTS_E_ARG. */
int qtts_safetensors_open(const char *path, qtts_safetensors **out);
/* The tensors of the file, in header order: count, then name i. */
int qtts_safetensors_count(qtts_safetensors *f, int *n);
int qtts_safetensors_name(qtts_safetensors *f, int i, char *buf, int len);
/* TSafeTensorsFile.Tensor (talker.pas:300): dtype (QTTS_DTYPE_F32, _BF16,
 * _F16 or _OTHER), ndim and shape[QTTS_MAX_DIMS], a pointer to its bytes in
 * the mapping (valid until close) and their count; NULL outputs skipped.  An
 * absent name is QTTS_E_ARG. */
int qtts_safetensors_tensor(qtts_safetensors *f, const char *name, int *dtype, int *ndim, int64_t *shape,
                            const void **data, int64_t *bytes);
int qtts_safetensors_close(qtts_safetensors *f);

/* QwenLmStack (lm.pas:174-179: TQwen3Model.CreateStack of the file, with
 * aPrefix "talker.model." or "talker.code_predictor.model."): the stack
 * from the tensors {prefix}layers.{i}.self_attn.{q,k,v,o}_proj.weight,
 * .self_attn.{q,k}_norm.weight, .mlp.{gate,up,down}_proj.weight,
 * .input_layernorm.weight, .post_attention_layernorm.weight and
 * {prefix}norm.weight.  Matrices F32 or BF16 (read in place, converted on
 * the device to config->dtype as qtts_stack_create); norms widened to
 * float32 (QwenWiden, lm.pas:159-172).  A missing tensor or a shape other
 * than the config's is QTTS_E_ARG. */
int qtts_stack_create_safetensors(qtts_device *dev, const qtts_stack_config *config, qtts_safetensors *f,
                                  const char *prefix, qtts_stack **out);
/* TQwenLmHeads.Add (lm.pas:277-308) from the file's tensor `name`
 * ([rows][hidden], F32 or BF16, e.g. talker.codec_head.weight,
 * talker.code_predictor.lm_head.{g}.weight). */
int qtts_heads_add_safetensors(qtts_heads *heads, qtts_safetensors *f, const char *name, int rows, int *index);
/* The cached blob of a stack: its weights as held on the device (F32 rows
 * or row-packed Q8_0), its config and norms, and a crc32c of the whole,
 * written to `path` (through path.tmp, then renamed) ... */
int qtts_stack_save(const qtts_stack *stack, const char *path);
/* ... and read back without a conversion.  Not a blob of this build
 * (magic, dimensions, size) or a checksum mismatch: QTTS_E_ARG. */
int qtts_stack_load(qtts_device *dev, const char *path, qtts_stack **out);

/* ------------------------------------------------------------------ the 12 Hz codec */

/* TQwenCodec.Create (src/tts/mormot.ai.tts.qwen.codec.pas:644-731): the
 * decoder of the speech_tokenizer checkpoint (its model.safetensors, F32 or
 * BF16 tensors under the reference's names: decoder.quantizer.*,
 * decoder.pre_conv.*, decoder.pre_transformer.*, decoder.upsample.*,
 * decoder.decoder.*) on the device.  A missing tensor or a shape other than
 * the reference's is QTTS_E_ARG. */
int qtts_codec_create_safetensors(qtts_device *dev, qtts_safetensors *f, qtts_codec **out);
/* TQwenCodec.Reset (codec.pas:776-792): the next frame starts a sentence. */
int qtts_codec_reset(qtts_codec *c);
/* TQwenCodec.Decode (codec.pas:1019-1038): codes[frames][16] (host) ->
 * pcm[frames * 1920] (host) in [-1, 1]; frames of successive calls follow
 * each other.  A code >= 2048 is QTTS_E_ARG (negative codes read as 0);
 * at most 2048 frames a call. */
int qtts_codec_decode(qtts_codec *c, const int32_t *codes, int frames, float *pcm);
/* TQwenCodec.Frames: the frames decoded since the last reset. */
int qtts_codec_frames(qtts_codec *c, int64_t *frames);
int qtts_codec_destroy(qtts_codec *c);

/* ------------------------------------------------------------------ talkers (batched frames) */

typedef struct qtts_talkers qtts_talkers;

/* TQwenTalker (talker.pas:78-158), greedy, for many utterances at once: the
 * per-frame loop of NextFrame (talker.pas:640-681) over a talker batch and a
 * predictor batch (not owned; heads as for qtts_talker_create).  No
 * counterpart object in the reference, which runs one TQwenTalker per
 * utterance; each utterance follows that protocol exactly.  Utterance ids
 * are the talker batch's sequence ids; the predictor batch needs as many
 * sequences, `groups` positions and 2 rows per sequence per call.  A frame
 * of n utterances is 15 batched predictor calls and one batched talker call
 * (tcgen05 projections, paged KV), with the choices on the device. */
int qtts_talkers_create(qtts_batch *talker, qtts_batch *predictor, const qtts_talker_config *config,
                        const float *codec_emb, const float *pred_emb, qtts_talkers **out);
/* The end of TQwenTalker.Start (talker.pas:561-592) for nseq utterances
 * seqs[i] (distinct), in one batched prefill: talker Reset + Forward of
 * rows[i] rows (all concatenated in prefill [sum rows][hidden]), the
 * utterance's trailing text rows (trailing_rows[i] rows, concatenated in
 * trailing; trailing_rows may be NULL for none), tts_pad [hidden] after
 * them, empty history, ChooseCode0 of frame 0. */
int qtts_talkers_start(qtts_talkers *t, int nseq, const int32_t *seqs, const int32_t *rows, const float *prefill,
                       const int32_t *trailing_rows, const float *trailing, const float *tts_pad);
/* TQwenTalker.Start from token ids (as qtts_talker_start_prompt) for nseq
 * utterances seqs[i] at once, every prompt row built on the device in one
 * text projection: utterance i's ids (n_ids[i] of them) and codec ids
 * (n_codec[i]) follow those of the utterances before it in ids / codec;
 * non_streaming[i] (NULL: all streaming).  Then as qtts_talkers_start. */
int qtts_talkers_start_prompt(qtts_talkers *t, qtts_textproj *tp, const qtts_prompt_tokens *tok, int nseq,
                              const int32_t *seqs, const int32_t *ids, const int32_t *n_ids, const int32_t *codec,
                              const int32_t *n_codec, const int32_t *non_streaming);
/* TQwenTalker.NextFrame (talker.pas:640-681) for nseq started utterances
 * seqs[i] (distinct): codes [nseq][groups] receives row i's frame and
 * more[i] = 1, or more[i] = 0 when the utterance has chosen eos (its codes
 * row untouched). */
int qtts_talkers_next_frame(qtts_talkers *t, int nseq, const int32_t *seqs, int32_t *codes, int32_t *more);
/* The CUDA stream (cudaStream_t) the frames run on, for callers that time
 * them with events. */
int qtts_talkers_stream(qtts_talkers *t, void **stream);
/* The talker probes of TQwenTalker.Emit (talker.pas:590, 678) for utterance
 * seq: the logits (head 0, [vocab]) and the normed state ([hidden]) of its
 * last talker forward.  seq must have taken part in the last talker call of
 * this object (qtts_talkers_start or _next_frame), else QTTS_E_STATE.
 * Either pointer may be NULL. */
int qtts_talkers_probe(qtts_talkers *t, int seq, float *logits, float *hidden);
int qtts_talkers_destroy(qtts_talkers *t);
/* The sampling of every utterance of the batch (TQwenSampling as for
 * qtts_talker_set_sampling): utterance s draws from the stream seed + s, so
 * that it picks the codes a lone qtts_talker with seed + s would pick from
 * the same logits.  The first code 0 is drawn by qtts_talkers_start: set it
 * before. */
int qtts_talkers_set_sampling(qtts_talkers *t, const qtts_sampling *s);

/* ------------------------------------------------------------------ utilities */

/* InferQuantizeRowQ8_0Ref (mormot2-ai, used at lm.pas:267): n float32 (n %
 * 32 == 0) to n/32 ggml blocks of 34 bytes, computed on the device. */
int qtts_quantize_q8_0(qtts_device *dev, const float *src, int64_t n, uint8_t *dst);

/* The message of the last failure on this thread ("" if none). */
const char *qtts_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* QTTS_H */
