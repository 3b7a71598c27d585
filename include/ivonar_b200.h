/*
 * ivonar_b200.h — C ABI of libivonar_b200.so, the sm_100a implementation of the
 * Ivonar ternary token loop (decode step, prompt prefill, sampler).
 *
 * Every pointer named "device" is CUDA device memory owned by the caller (the
 * Python host allocates it with torch). Streams are passed as `void*` holding a
 * cudaStream_t. Every entry point returns 0 on success or an IVB_E* code; the
 * message of the last failure on the calling thread is ivb_last_error().
 * Nothing here allocates device memory: the decoder asks for a workspace size
 * and the caller hands in the buffer.
 *
 * Weight format (unchanged from the reference checkpoint, q2_g128):
 *   packed [rows][row_bytes] uint8: input 4j+f sits in bits 2f..2f+1 of byte j,
 *          code = ternary value + 1 in {0,1,2}; row_bytes = ceil(in/4) padded to 16.
 *   scales [rows][scale_stride] fp16: one positive scale per 128 inputs.
 *   bias   [rows] fp32 or NULL.
 * Reference: src/ivonar_inference/quantization.py:13-32 (unpack/dequantize),
 * kernel_decoder.py:84-142 (Matrix: row concatenation/interleave, 16-byte rows).
 */
#ifndef IVONAR_B200_H
#define IVONAR_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IVB_ABI_VERSION 2

enum {
  IVB_OK = 0,
  IVB_EINVAL = 1,       /* bad argument or unsupported shape */
  IVB_ECUDA = 2,        /* a CUDA runtime call failed */
  IVB_ETIMEOUT = 3,     /* a bounded inter-CTA wait ran out (device error word) */
  IVB_ECAPACITY = 4,    /* the decoder has no free position left */
  IVB_EUNSUPPORTED = 5  /* the device cannot run this build (not sm_100) */
};

/* GEMV epilogues (reference ternary.cu:53 EPI_STORE / EPI_RESIDUAL / EPI_SILU_PAIR). */
enum { IVB_EPI_STORE = 0, IVB_EPI_RESIDUAL = 1, IVB_EPI_SILU_PAIR = 2 };

/* Mixer kinds (reference config.py layer_types "mamba" / "mla"). */
enum { IVB_MAMBA = 0, IVB_MLA = 1 };

/* decode run flags */
enum {
  IVB_RUN_SAMPLE = 1,       /* sample a token after every step (reference StaticDecoder._step + _sample) */
  IVB_RUN_SAMPLE_ONLY = 2,  /* sample from the current logits without a step (reference StaticDecoder.sample) */
  IVB_RUN_HEAD_ALL = 4      /* compute logits on every fed step, not only the last one */
};

/* One ternary projection (or a row-stack of several) in device memory. */
typedef struct IvbTernary {
  const uint8_t* packed;
  const uint16_t* scales;
  const float* bias;
  int32_t rows;
  int32_t in_features;
  int32_t row_bytes;
  int32_t scale_stride;
} IvbTernary;

/* One residual block. Reference: model.py:32-35 (IvonarBlock.forward),
 * recurrent.py:41-139 (RecurrentMixer), attention.py:75-151 (LatentAttention). */
typedef struct IvbLayerDesc {
  int32_t kind;               /* IVB_MAMBA or IVB_MLA */
  const float* mixer_norm;    /* [hidden] RMSNorm weight */
  float mixer_norm_eps;
  const float* ffn_norm;      /* [hidden] */
  float ffn_norm_eps;
  IvbTernary entry;           /* mamba: [in_proj ; bc_dt_proj]   mla: [q_proj ; kv_down_proj ; k_rope_proj] */
  IvbTernary out;             /* out_proj */
  IvbTernary gate_up;         /* gate_proj and up_proj rows interleaved (2r = gate r, 2r+1 = up r) */
  IvbTernary down;            /* down_proj */
  /* mamba (RecurrentMixer) */
  const float* decay;         /* [heads, state] = -softplus(log_decay) */
  const float* theta;         /* [heads, state] */
  const float* skip;          /* [heads * head_dim] */
  const float* conv_weight;   /* [hidden, conv_taps] */
  const float* conv_bias;     /* [hidden] */
  float* ssm_state;           /* [heads, state, head_dim, 2] fp32 (complex) */
  float* prev_force;          /* [heads, state, head_dim] */
  float* conv_state;          /* [hidden, conv_taps - 1] */
  int32_t conv_taps;
  float half_dt_min;          /* 0.5 * dt_min */
  float half_dt_range;        /* 0.5 * (dt_max - dt_min) */
  /* mla (LatentAttention) over the compressed latent cache */
  IvbTernary k_nope_up;       /* [heads * nope, latent] (absorbed into the query) */
  IvbTernary v_up;            /* [hidden, latent]       (applied after the softmax) */
  const float* rope;          /* [max_len, rope_dim / 2, 2] (cos, sin) */
  int8_t* latent_q;           /* cache [max_len, latent] int8 codes of the quantised latent */
  float* latent_scale;        /* cache [max_len] per-position activation scale */
  uint16_t* k_rope_cache;     /* cache [heads, max_len, rope_dim padded to 8] fp16 rotated k_rope */
  float attn_scale;           /* 1 / sqrt(head_dim) */
  /* mla: the decompressed cache the decode kernel attends over (rows of head_dim rounded up to 4 floats,
   * zero padded; 16-byte aligned). Keys: k_nope = W_k(latent) + b_k, then the rotated k_rope as stored
   * in k_rope_cache; values: W_v(latent) + b_v. The single-sequence decoder and its prefill write them;
   * null in descriptions used only by the batched kernels. */
  float* k_cache;             /* [heads, max_len, head_dim padded to 4] fp32 */
  float* v_cache;             /* [heads, max_len, head_dim padded to 4] fp32 */
} IvbLayerDesc;

/* The whole model plus the decoder state buffers. Reference: kernel_decoder.py:179-283. */
typedef struct IvbModelDesc {
  int32_t abi_version;        /* IVB_ABI_VERSION */
  int32_t vocab, hidden, heads, head_dim, state_dim, latent_dim, rope_dim, nope_dim, dense;
  int32_t num_layers, max_len, max_top_k;
  float act_eps;              /* activation quantiser floor (TernaryLinear eps, 1e-5) */
  float norm_clip;            /* RMSNorm clip (8.0) */
  IvbTernary head;            /* tied token embedding / LM head [vocab, hidden] */
  const float* final_norm;
  float final_norm_eps;
  const IvbLayerDesc* layers; /* host array [num_layers] */
  /* state (device) */
  float* logits;              /* [vocab] */
  int64_t* token;             /* [1] last fed or sampled token */
  int64_t* position;          /* [1] next cache slot */
  uint8_t* seen;              /* [vocab] repetition-penalty flags (torch.bool) */
  int64_t* history;           /* [history_len] tokens sampled by the last run */
  int32_t history_len;
  const float* sampling;      /* [3] temperature, penalty, inverse_penalty */
  const int64_t* top_k;       /* [1] */
  uint64_t* rng;              /* [2] philox key (seed), draw counter */
} IvbModelDesc;

typedef struct IvbDecoder IvbDecoder; /* host-side plan; opaque */

/* ---- batched decode (independent sequences, one token each per step) ---------------------------- */
/* Per-layer recurrent state and latent caches of `batch` sequences: the pointers of sequence 0, the
 * sequences following contiguously with the sizes of the single-sequence layout (ssm_state
 * heads*state*head_dim*2 floats, prev_force heads*state*head_dim, conv_state hidden*(conv_taps-1),
 * latent_q max_len*latent_pad bytes, latent_scale max_len floats, k_rope_cache heads*max_len*rope_pad
 * halves, with latent_pad = latent rounded up to 16 and rope_pad = rope_dim rounded up to 8). */
typedef struct IvbBatchLayer {
  float* ssm_state;
  float* prev_force;
  float* conv_state;
  int8_t* latent_q;
  float* latent_scale;
  uint16_t* k_rope_cache;
} IvbBatchLayer;

typedef struct IvbBatch {
  int32_t batch;
  const IvbBatchLayer* layers; /* host array [num_layers] */
  int64_t* tokens;             /* [batch] token of each sequence fed this step; replaced by the sampled one */
  int64_t* positions;          /* [batch] cache slot of that token; advanced by one per step */
  float* logits;               /* [batch][vocab] */
  uint8_t* seen;               /* [batch][vocab] repetition-penalty flags */
  uint64_t* rng;               /* [batch][2] philox key (per-sequence seed), draw counter */
  int64_t* history;            /* [batch][history_len] sampled tokens (may be NULL) */
  int32_t history_len;
  int32_t* step;               /* [1] device step counter: the step that runs writes column *step, then
                                  advances it (the caller zeroes it at the start of a generation) */
  const float* sampling;       /* [3] temperature, penalty, inverse_penalty (shared) */
  const int64_t* top_k;        /* [1] (shared) */
} IvbBatch;

/* ---- library ---------------------------------------------------------------------------------- */
int32_t ivb_abi_version(void);
const char* ivb_last_error(void);
/* 1 when the current CUDA device is an sm_100 part this build runs on. */
int32_t ivb_device_supported(void);

/* ---- unit entry points (each one a single kernel launch) ------------------------------------- */

/* Per-token int8 activation quantiser with optional fused RMSNorm (clip, then weight).
 * Replaces ternary.cu:148-197 quantize_source and quantization.py:35-38 quantize_activations.
 * q8 [n] natural order, *scale = max(amax/127, act_eps), xsum [ceil(n/64)] chunk sums (may be NULL). */
int32_t ivb_quantize(const float* x, const float* norm_weight, int32_t n, float norm_eps, float norm_clip,
                     float act_eps, int8_t* q8, float* scale, int32_t* xsum, void* stream);

/* Exact integer core of the ternary GEMV: dots[r][g] = sum over the 128 inputs of group g of
 * (code-1) * q8. Replaces the integer part of ternary.cu:241-258 chunk_dot (dot - xsum). */
int32_t ivb_ternary_group_dots(const IvbTernary* m, const int8_t* q8, int32_t* dots, void* stream);

/* Fused (RMSNorm +) quantise + ternary GEMV + epilogue, one launch over all rows.
 * norm_weight == NULL: plain quantisation. Replaces ternary.cu:356-388 gemv_* entry points. */
int32_t ivb_ternary_gemv(const IvbTernary* m, const float* x, const float* norm_weight, float norm_eps,
                         float norm_clip, float act_eps, int32_t epilogue, float* out, void* stream);

/* Prefill quantiser for `rows` token rows: x [rows][n] fp32 (RMSNorm first when norm_weight is given) ->
 * q8 int8 in the tiled GEMM activation layout, scale [rows], and, when gsum is not NULL,
 * gsum [rows][ceil(n/128)] int32 sums of the codes per 128-input group. ldq: a multiple of 128, at
 * least n (inputs n..ldq-1 are written as zero).
 * Tiled layout: one 16384-byte block per (token tile t/128, input group i/128) at
 * ((t/128) * (ldq/128) + i/128) * 16384; inside it, the 16-input chunk k = (i%128)/16 of token row
 * r = t%128 sits at (8*(r/8) + k) * 128 + (r%8) * 16, and within the chunk byte 4f+b holds input 4b+f.
 * q8 must hold ceil(rows/128) * 128 * ldq bytes (16-byte aligned); the pad rows of the last tile are
 * not written. Replaces ternary.cu:637-668 quantize_tile_*. */
int32_t ivb_quantize_rows(const float* x, int32_t rows, int32_t n, const float* norm_weight, float norm_eps,
                          float norm_clip, float act_eps, int8_t* q8, int32_t ldq, float* scale, int32_t* gsum,
                          void* stream);

/* Prefill ternary GEMM on tcgen05 int8 MMA (weights as signed codes in TMEM, activations from shared
 * memory, TMEM accumulators), `rows_t` tokens at once:
 * out[t][r] = epilogue(scale[t] * sum_g s[r][g] * (sum_{k in g} (code[r][k] - 1) * q8[t][k]) + bias[r])
 * with q8 (tiled layout, same ldq)/scale from ivb_quantize_rows; out row stride ldo (SILU_PAIR writes
 * rows/2 outputs per token). Uses all 512 TMEM columns of the SMs it runs on.
 * *error becomes IVB_ETIMEOUT if a bounded wait on the tensor core ran out. Replaces ternary.cu:688-783.
 * Few tokens (too few row x token tiles to fill the GPU) split the inputs across CTAs; the split
 * partial sums of this entry point live in a file-scope device scratch (16 MB) shared by every call on
 * the device, so calls on one device must not overlap in time: issue them on one stream or order them
 * with events. ivb_decoder_prefill and ivb_batch_decode keep their partial sums in their own workspace
 * and share nothing. */
int32_t ivb_ternary_gemm(const IvbTernary* m, const int8_t* q8, int32_t ldq, const float* act_scale, int32_t rows_t,
                         int32_t epilogue, float* out, int32_t ldo, uint32_t* error, void* stream);

/* Split-K variant of ivb_ternary_gemv (same arguments, same results within fp32 rounding): the input
 * columns are spread over more CTAs, each column block's partial row sums go to a static device
 * scratch, and a second kernel adds them in column-block order, so two calls on the same inputs give
 * the same bits. It has no counterpart in the reference. It is for callers that may not allocate
 * device memory at call time: a serving process whose pool already holds the GPU's memory (a
 * cudaMalloc there fails or waits for the whole device), or code on a latency-bound path where
 * cudaMalloc's implicit device synchronisation is not acceptable. It allocates nothing: the scratch is
 * a file-scope __device__ array of 16 column blocks x 32768 fp32 row sums (rows > 32768 or
 * in_features > 16384 return IVB_EINVAL); its address is looked up, and the kernel's shared-memory
 * limit set, once per device on the first call with that device current, so make the first call on
 * each device outside any stream capture. The cached address belongs to the device's primary context:
 * do not use the library across a cudaDeviceReset. Calls that overlap in time on one device (other
 * streams or threads) share the scratch and race: serialise them. */
int32_t ivb_ternary_gemv_splitk(const IvbTernary* m, const float* x, const float* norm_weight, float norm_eps,
                                float norm_clip, float act_eps, int32_t epilogue, float* out, void* stream);

/* Sampler over one logits row: temperature, repetition penalty, exact top-k, softmax and an
 * inverse-CDF draw with a Philox4x32-10 uniform (key rng[0], counter rng[1]++).
 * Replaces ternary.cu:1064-1337 logit_bounds + sample_token. token/history: int64 [1] each. */
int32_t ivb_sample(const float* logits, uint8_t* seen, int32_t vocab, const float* sampling,
                   const int64_t* top_k, int32_t max_top_k, uint64_t* rng, int64_t* token, int64_t* history,
                   void* stream);

/* Batched decode: `steps` tokens for every sequence of `b` (each step: the decoder's layers over all
 * sequences at once as tcgen05 GEMMs, per-sequence SSM step / latent-cache append / attention, head
 * GEMM, per-sequence sampler). The decoder handle supplies the weights and shapes; its own
 * single-sequence state is not touched. Workspace: ivb_batch_workspace_bytes, 256-byte aligned.
 * Replaces StaticDecoder's batch_size > 1 step (decoder.py:67,96,387-394); the reference GPU kernels
 * have no batched decode. */
uint64_t ivb_batch_workspace_bytes(const IvbDecoder* dec, int32_t batch);
int32_t ivb_batch_decode(IvbDecoder* dec, const IvbBatch* b, int32_t steps, void* workspace, uint64_t workspace_bytes,
                         void* stream);

/* Unit steps of the batched decode for callers that orchestrate the layers themselves (tensor-parallel
 * shards: `channels` = heads * head_dim of the shard, the entry rows laid out as the shard's
 * [value | gate | B, C, dt per head] or [q | latent | k_rope]):
 * ivb_batch_embed: resid[b] = embedding row of tokens[b] (advances *step_counter when not NULL);
 * ivb_batch_ssm: one SSM step per sequence (recurrent_step, ternary.cu:421-482);
 * ivb_batch_mla: latent-cache append at positions[b] and absorbed attention (ternary.cu:509-611);
 * ivb_batch_sample: per-sequence sampler, then positions[b] += 1 (ternary.cu:1099-1337). */
int32_t ivb_batch_embed(const IvbTernary* head, const int64_t* tokens, int32_t batch, int32_t hidden, float* resid,
                        int32_t* step_counter, void* stream);
int32_t ivb_batch_ssm(const IvbLayerDesc* layer, const IvbBatchLayer* state, const float* ent, int32_t ld, int32_t batch,
                      int32_t channels, int32_t heads, int32_t head_dim, int32_t state_dim, float* y, void* stream);
int32_t ivb_batch_mla(const IvbLayerDesc* layer, const IvbBatchLayer* state, const float* ent, int32_t ld,
                      const int64_t* positions, int32_t batch, int32_t channels, int32_t latent, int32_t heads,
                      int32_t head_dim, int32_t rope, int32_t nope, int32_t max_len, float act_eps, uint32_t* error,
                      float* y, void* stream);
int32_t ivb_batch_sample(const float* logits, uint8_t* seen, int32_t vocab, int32_t batch, const float* sampling,
                         const int64_t* top_k, int32_t max_top_k, uint64_t* rng, int64_t* tokens, int64_t* positions,
                         int64_t* history, int32_t history_len, const int32_t* step_counter, void* stream);

/* Checkpoint ingest: validation of a checkpoint's packed buffers once they are on the device, in one
 * launch (replaces the reference loader's chunked CPU checks, loader.py:94-112). Each buffer is a packed
 * ternary weight array (uint8, kind IVB_CHECK_PACKED: the reserved 2-bit code 3 is an error) or a g128
 * scale array (fp16, kind IVB_CHECK_SCALES: every scale finite and positive). `buffers` is a device
 * array of `count` descriptors; bad[0..2] (device int32) receive the lowest index of a buffer holding
 * code 3, a non-finite scale, a non-positive scale, or `count` when none does. Asynchronous on
 * `stream` (the caller reads bad after synchronising). */
#define IVB_CHECK_PACKED 0
#define IVB_CHECK_SCALES 1
typedef struct IvbCheckBuffer {
  const void* data;
  int64_t count;              /* bytes (packed) or fp16 values (scales) */
  int32_t kind;               /* IVB_CHECK_PACKED or IVB_CHECK_SCALES */
  int32_t pad;
} IvbCheckBuffer;
int32_t ivb_validate_buffers(const IvbCheckBuffer* buffers, int32_t count, int32_t* bad, void* stream);

/* Vocabulary-sharded sampling (tensor parallel, head rows split over the ranks). ivb_batch_topk_slice:
 * per sequence, the top min(K, vloc) candidates of this rank's slice [v0, v0 + vloc) of the vocabulary
 * (logits and repetition flags [batch][vloc]) by (score key desc, id asc), as the sampler's order-
 * preserving score keys and global ids in slots [0, kc) of keys / ids [batch][kc], padded with key 0
 * (kc >= min(max_top_k, vocab, 256)). ivb_batch_sample_merge: the gathered candidates of all ranks
 * ([world][batch][kc], rank-major, ranks' slices in vocabulary order) merged by the unsharded sampler's
 * selection, CDF and Philox draw, so every rank draws the token ivb_batch_sample would draw over the whole
 * vocabulary; then history (at step_counter - 1), position += 1, and the repetition flag when the token
 * lies in [v0, v0 + vloc). Replaces the replicated head + sampler of ternary.cu:374 (gemv_prequant_store)
 * and :1099-1337 (sample_token). */
int32_t ivb_batch_topk_slice(const float* logits, const uint8_t* seen, int32_t vloc, int32_t v0, int32_t vocab, int32_t batch,
                             const float* sampling, const int64_t* top_k, int32_t max_top_k, int32_t kc, uint32_t* keys,
                             int32_t* ids, void* stream);
int32_t ivb_batch_sample_merge(const uint32_t* keys, const int32_t* ids, int32_t world, int32_t batch, int32_t kc, int32_t vocab,
                               const int64_t* top_k, int32_t max_top_k, uint64_t* rng, int64_t* tokens, int64_t* positions,
                               int64_t* history, int32_t history_len, const int32_t* step_counter, uint8_t* seen, int32_t v0,
                               int32_t vloc, void* stream);

/* Per-row max |x| (rows x n fp32) into amax [rows]; with ivb_quantize_rows_amax the quantisation of a
 * row-parallel shard uses the amax of the whole row (after an all-reduce MAX), so every shard's codes
 * equal the unsharded quantiser's: scale = max(amax / 127, act_eps), code = rint(x / scale). */
int32_t ivb_rows_amax(const float* x, int32_t rows, int32_t n, float* amax, void* stream);
int32_t ivb_quantize_rows_amax(const float* x, int32_t rows, int32_t n, const float* amax, float act_eps, int8_t* q8,
                               int32_t ldq, float* scale, void* stream);

/* Unit probe of the decode kernel's GEMV row routine (the hot path of every projection op of
 * ivb_decoder_run; replaces the reference's gemv_prequant_store row loop, kernels/ternary.cu:302-354,
 * and the CPU decoder's row_dot, cpu_decoder.py:73-86). `stage` (device) is one weight-stream chunk:
 * [k rows x row_bytes packed q2 codes][k x scale_stride fp16 group scales, padded to 16 bytes]
 * [k fp32 biases when has_bias]; q8 (device) the in_n int8 activation codes. out[r] = act_scale *
 * sum_g scale[r][g] * sum_{j in g} (code[r][j] - 1) q8[j] (+ bias[r]), computed as in the decode kernel
 * (integer 64-input chunk dots, fp32 over the chunks): lanes_log = -1 runs the kernel's own choice of
 * routine for the shape; 0..5 the general routine with 2^lanes_log lanes per row. */
int32_t ivb_decode_rows(const uint8_t* stage, int32_t k, int32_t row_bytes, int32_t scale_stride, int32_t has_bias,
                        float act_scale, const int8_t* q8, int32_t in_n, int32_t lanes_log, float* out, void* stream);

/* Debug/failure-detection probe: one CTA waits for a barrier count that never arrives, with a
 * bounded spin of timeout_ns; returns IVB_ETIMEOUT and leaves the context usable. */
int32_t ivb_probe_wait_timeout(uint32_t* counter, uint32_t* error_word, uint64_t timeout_ns, void* stream);

/* ---- persistent decoder ----------------------------------------------------------------------- */
/* Replaces kernel_decoder.py KernelDecoder._build/_step/_capture_burst/advance_many: one persistent
 * cooperative kernel runs every layer, the head and the sampler for `steps` tokens per launch. */
int32_t ivb_decoder_create(const IvbModelDesc* desc, int32_t ctas, IvbDecoder** out);
void ivb_decoder_destroy(IvbDecoder* dec);
uint64_t ivb_decoder_workspace_bytes(const IvbDecoder* dec);
int32_t ivb_decoder_num_phases(const IvbDecoder* dec);
int32_t ivb_decoder_ctas(const IvbDecoder* dec);
/* Uploads the phase program into the caller's workspace (device, >= workspace_bytes, 256-aligned). */
int32_t ivb_decoder_bind(IvbDecoder* dec, void* workspace, void* stream);
/* Run `steps` tokens. feed == NULL: each step consumes the token sampled by the previous one
 * (requires IVB_RUN_SAMPLE). feed != NULL: device int64 [steps] teacher-forced tokens.
 * timeout_ns bounds every inter-CTA wait (0 = 1 s). Asynchronous; errors surface through
 * ivb_decoder_check. */
int32_t ivb_decoder_run(IvbDecoder* dec, int32_t steps, const int64_t* feed, int32_t flags, uint64_t timeout_ns,
                        void* stream);
/* Device timeline for tuning: while `buffer` (device uint64 [num_phases][ctas][8]) is set, each run
 * records the globaltimer (ns) of step `step`, per phase and CTA: [0] work start, [1..6] marks inside
 * the phase (0 where a phase has fewer), [7] work end before the phase's barrier. NULL turns it off. */
int32_t ivb_decoder_trace(IvbDecoder* dec, uint64_t* buffer, int32_t step);
/* Device workspace (bytes) for one ivb_decoder_prefill call of up to max_tokens tokens. */
uint64_t ivb_decoder_prefill_workspace_bytes(const IvbDecoder* dec, int32_t max_tokens);
/* Prompt prefill with all `count` tokens per layer at once: device int64 tokens [count] at positions
 * start_position.. (tcgen05 GEMMs for every projection, recurrent scan over the tokens, latent/k_rope
 * cache fill and causal latent attention), then the head of the last token into logits; leaves caches,
 * recurrent state, position and token where token-by-token decoding would. Chunked prompts: call again
 * with the next tokens and start_position advanced (the recurrent state carries over). Asynchronous.
 * Replaces kernel_decoder.py:457-479 prefill and ternary.cu:688-982 (tile GEMM/recurrence/attention). */
int32_t ivb_decoder_prefill(IvbDecoder* dec, const int64_t* tokens, int32_t count, int32_t start_position, void* workspace,
                            uint64_t workspace_bytes, void* stream);
/* Synchronises the stream and returns IVB_ETIMEOUT/IVB_ECAPACITY if the device error word is set. */
int32_t ivb_decoder_check(IvbDecoder* dec, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IVONAR_B200_H */
