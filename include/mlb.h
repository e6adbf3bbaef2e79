/*
 * mini_llama_b200 — C ABI of the B200 (sm_100a) implementation of mini_llama's
 * decode/prefill hot path.
 *
 * Plain pointers, sizes and int status codes; no C++ or torch types.  Every
 * entry point that replaces a reference interface cites it as
 * "replaces <reference file>:<lines>" (paths inside the mini_llama project).
 * The C++17 adapter in mini_llama_b200/adapter/ implements the reference's own
 * headers (include/cuda_quant.h, cuda_attention.h, cuda_ops.h, cuda_kv_cache.h,
 * cuda_tensor.h, cuda_data.h) on top of these functions, so the reference's
 * forward.cpp, loaders and sampler link against this library unchanged.
 *
 * Conventions
 *  - All device pointers belong to `device`.  Unless stated otherwise a call
 *    only enqueues work on the library stream of that device (see
 *    mlb_get_stream) and returns; results are visible to later calls of this
 *    library, to mlb_memcpy_d2h and after mlb_synchronize.
 *  - Tensors are fp32, row-major.  Quantized weights are GGUF blocks of 32
 *    elements, rows of ceil(K/32) blocks: Q8_0 {fp16 d; int8 q[32]} (34 B),
 *    Q4_0 {fp16 d; uint8 q[16]} (18 B, w = d*(q-8), low nibbles are elements
 *    0-15), Q4_1 {fp16 d; fp16 m; uint8 q[16]} (20 B, w = d*q + m).
 *  - KV caches are fp32 [n_layers, max_seq_len, n_kv_heads, head_dim].
 *  - On failure a call returns a nonzero mlb_status and mlb_last_error()
 *    returns the message (thread-local), prefixed with the caller's name the
 *    way the reference's exceptions are.
 */
#ifndef MINI_LLAMA_B200_MLB_H
#define MINI_LLAMA_B200_MLB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MLB_ABI_VERSION 1

typedef enum {
    MLB_OK = 0,
    MLB_ERR_INVALID_ARGUMENT = 1, /* the reference throws std::runtime_error */
    MLB_ERR_OUT_OF_RANGE = 2,     /* the reference throws std::out_of_range */
    MLB_ERR_CUDA = 3,             /* CUDA runtime error */
    MLB_ERR_UNSUPPORTED = 4,      /* shape outside what this build supports */
    MLB_ERR_DEVICE_TIMEOUT = 5    /* a bounded device-side wait expired */
} mlb_status;

typedef enum { MLB_F32 = 0, MLB_Q8_0 = 1, MLB_Q4_0 = 2, MLB_Q4_1 = 3 } mlb_qtype;
typedef enum { MLB_ROPE_NORMAL = 0, MLB_ROPE_NEOX = 1 } mlb_rope_type;

const char* mlb_last_error(void);
int mlb_abi_version(void);

/* ------------------------------------------------------------ device runtime
 * replaces include/cuda_data.h:16-35 (CheckCudaRuntimeBuilt, GetCudaDeviceCount,
 * CudaSetDevice, GetCudaDeviceInfo, CudaMallocBytes, CudaFreeBytes,
 * CudaMemcpyBytes) and the storage of include/cuda_tensor.h:9-58.
 * mlb_malloc/mlb_free are stream-ordered on the library stream and served from
 * a per-device pool that keeps freed blocks (no cudaFree in steady state). */
typedef struct {
    char name[256];
    int compute_major;
    int compute_minor;
    size_t total_memory_bytes;
    int sm_count;
    int driver_version;
    int runtime_version;
} mlb_device_info;

int mlb_device_count(int* count);
int mlb_set_device(int device);
int mlb_get_device_info(int device, mlb_device_info* info);
int mlb_get_stream(int device, void** cuda_stream);
int mlb_malloc(int device, size_t bytes, void** ptr);
int mlb_free(int device, void* ptr);
/* host -> device: returns once the host buffer may be reused */
int mlb_memcpy_h2d(int device, void* dst, const void* src, size_t bytes);
/* device -> host: waits for prior library work on the device, then copies */
int mlb_memcpy_d2h(int device, void* dst, const void* src, size_t bytes);
int mlb_memcpy_d2d(int device, void* dst, const void* src, size_t bytes);
int mlb_memset(int device, void* dst, int value, size_t bytes);
int mlb_synchronize(int device);

/* ------------------------------------------------------------ quantized linear
 * y[rows, out] = x[rows, in] . dequant(W[out, in])^T (+ bias[out])
 * replaces include/cuda_quant.h:13-38 (CudaQ80/Q40/Q41 Linear, ...DeviceWeight,
 * ...DeviceInput), reference kernels src/cuda_quant.cu:40-135.
 * block_count must equal out * ceil(in/32) (the reference's check,
 * src/cuda_quant.cu:175-181).  bias may be NULL.  rows <= 8 runs a
 * bandwidth-bound GEMV over the blocks (the integer tensor-core one on
 * matrices with many 16-row tiles, such as an lm_head; launches of it are
 * ordered on the library's stream, which its tile scheduler relies on);
 * 9..64 rows an integer-MMA linear (x's exact digit planes against the raw
 * quants) where it is the faster one, other batches the tcgen05 tensor-core
 * linear. */
int mlb_q80_linear(int device, const float* x, const void* w, size_t block_count, int rows,
                   int in_features, int out_features, const float* bias, float* y);
int mlb_q40_linear(int device, const float* x, const void* w, size_t block_count, int rows,
                   int in_features, int out_features, const float* bias, float* y);
int mlb_q41_linear(int device, const float* x, const void* w, size_t block_count, int rows,
                   int in_features, int out_features, const float* bias, float* y);
/* Same with the block type as an argument (MLB_Q8_0 / MLB_Q4_0 / MLB_Q4_1). */
int mlb_quant_linear(int device, int qtype, const float* x, const void* w, size_t block_count,
                     int rows, int in_features, int out_features, const float* bias, float* y);

/* F32 linear and matmul: replace include/cuda_matmul.h:11-33 (CudaLinear,
 * CudaLinearDeviceWeight, CudaLinearDeviceInput, CudaMatmul; the reference
 * calls cublasSgemm with a new handle per call, src/cuda_matmul.cpp:118-229).
 * mlb_f32_linear: y[rows, out] = x[rows, in] . W[out, in]^T (+ bias[out]).
 * mlb_f32_matmul: c[m, n] = a[m, k] . b[k, n], all row-major. */
int mlb_f32_linear(int device, const float* x, const float* w, int rows, int in_features,
                   int out_features, const float* bias, float* y);
int mlb_f32_matmul(int device, const float* a, const float* b, int m, int k, int n, float* c);

/* Prepared Q8_0 weights ("R16" layout): the same bytes regrouped into 16-row
 * tiles of 544-byte chunks (16 x 32 int8 quants, then 16 fp16 scales), every
 * chunk 16-byte aligned.  A caller that keeps a prepared copy gets the
 * tensor-core GEMV, which computes each block's dot product exactly in int32
 * (x split into three int8 digit planes per 32-element block) and applies the
 * scales in fp32.  No reference counterpart: the reference reads the GGUF
 * blocks in place; this is the layout its weights take inside the decode
 * session.  mlb_r16_bytes returns the size of the prepared copy (rows padded
 * to a multiple of 16). */
size_t mlb_r16_bytes(int rows, int cols);
int mlb_q80_repack_r16(int device, const void* w, int rows, int cols, void* w_r16);
int mlb_q80_linear_r16(int device, const float* x, const void* w_r16, int rows, int in_features,
                       int out_features, const float* bias, float* y);

/* ------------------------------------------------------------ quantization
 * Device quantizer, bit-identical to the reference's QuantizeToQ80 and
 * QuantizeToQ40 (src/quant.cpp:104-240, fp16 rounding of src/quant.cpp:17-52)
 * and, for Q4_1, to the reference GPU test's quantizer
 * (test/gpu_core_test.cpp:156-198).  replaces the host-side
 * QuantizeModelToQ80/Q40 (src/model.cpp:454-493) for weights already in HBM.
 * mlb_dequantize replaces DeQuantizeFromQ80/Q40, DequantizeFromQ41
 * (src/quant.cpp:153-317). */
int mlb_quantize(int device, int qtype, const float* x, int rows, int cols, void* blocks);
int mlb_dequantize(int device, int qtype, const void* blocks, int rows, int cols, float* y);

/* ------------------------------------------------------------ element-wise ops
 * replaces include/cuda_ops.h:11-46, reference kernels src/cuda_ops.cu:22-172 */
int mlb_rmsnorm(int device, const float* x, const float* weight, int n, float eps, float* y);
/* RoPE in place on q [n_heads, head_dim] and k [n_kv_heads, head_dim] at
 * position pos.  The rotation angles are the reference CPU's table values
 * (src/context.cpp:16-25: freq = 1/powf(theta, 2i/head_dim), angle = pos*freq)
 * computed on the host; rope_type MLB_ROPE_NORMAL pairs (2i, 2i+1),
 * MLB_ROPE_NEOX pairs (i, i + head_dim/2) (src/ops.cpp:123-168). */
int mlb_rope(int device, float* q, float* k, int n_heads, int n_kv_heads, int head_dim, int pos,
             float theta, int rope_type);
int mlb_silu(int device, const float* x, size_t n, float* y);
int mlb_mul(int device, const float* a, const float* b, size_t n, float* y);
int mlb_add(int device, const float* a, const float* b, size_t n, float* y);
int mlb_softmax(int device, const float* x, int n, float* y);
int mlb_embedding(int device, const float* table, int vocab_size, int dim, int token, float* y);
/* Index of the first maximum of x[n] (src/ops.cpp:199-212), written to the
 * device int at out_index. */
int mlb_argmax(int device, const float* x, int n, int* out_index);

/* ------------------------------------------------------------ KV cache
 * replaces CudaKVCache::WriteDevice (src/cuda_kv_cache.cpp:157-182): k and v
 * [n_kv_heads, head_dim] written at (layer, pos) of both caches by one kernel. */
int mlb_kv_write(int device, float* key_cache, float* value_cache, int n_layers,
                 int max_seq_len, int n_kv_heads, int head_dim, int layer, int pos,
                 const float* k, const float* v);

/* ------------------------------------------------------------ decode attention
 * out[n_heads, head_dim] = softmax(q . K[0..pos]^T / sqrt(head_dim)) . V[0..pos]
 * for query head h reading KV head h / (n_heads / n_kv_heads).
 * replaces include/cuda_attention.h:10-14 (CudaAttentionDecode,
 * CudaAttentionDecodeDeviceInputs), reference kernels
 * src/cuda_attention.cu:87-181.  Split-K over positions with a merged partial
 * softmax; scratch comes from the library's per-device workspace. */
int mlb_attention_decode(int device, const float* q, const float* key_cache,
                         const float* value_cache, int n_layers, int max_seq_len, int layer,
                         int pos, int n_heads, int n_kv_heads, int head_dim, float* out);
/* Batch of independent sequences: q [batch, n_heads, head_dim], caches
 * [batch, n_layers, max_seq_len, n_kv_heads, head_dim], positions[batch] a
 * device int array (each sequence attends to 0..positions[b]), out
 * [batch, n_heads, head_dim].  No reference counterpart: the reference decodes
 * one sequence per call; this is the batched form of the same computation. */
int mlb_attention_decode_batched(int device, int batch, const float* q, const float* key_cache,
                                 const float* value_cache, int n_layers, int max_seq_len,
                                 int layer, const int* positions, int max_pos, int n_heads,
                                 int n_kv_heads, int head_dim, float* out);

/* The same decode attention for callers that cannot allocate device memory
 * while decoding: for example an application in which another framework
 * already holds all free device memory, or a thread that must not take the
 * allocator's locks or risk the device synchronisation that freeing memory
 * can cause.  No counterpart in the reference.
 * The split-K partials live in one fixed 4 MiB array inside the library
 * image, present on every device that loads the library until the process
 * exits; a shape whose partials need more (n_heads x chunks x (head_dim + 2)
 * floats) is rejected with MLB_ERR_UNSUPPORTED.  The first call on a device
 * also does the library's one-time set-up for that device (its stream and the
 * array's device address), allocating no device memory; make that first call
 * before any stream capture.  Every call uses the same array, which keeps the
 * last call's contents; calls whose work overlaps on the GPU race on it.  This
 * library issues all of a device's work on one stream, so its own calls are
 * ordered. */
int mlb_attention_decode_noalloc(int device, const float* q, const float* key_cache,
                                 const float* value_cache, int n_layers, int max_seq_len,
                                 int layer, int pos, int n_heads, int n_kv_heads, int head_dim,
                                 float* out);

/* ------------------------------------------------------------ synthetic inputs
 * Seeded N(0, sigma) fill on the device, bit-identical to the host generator
 * used for fixtures (splitmix64 counter stream, Irwin-Hall sum of 12 uniform
 * 32-bit integers).  No reference counterpart (test and benchmark inputs). */
int mlb_synth_normal(int device, float* out, size_t n, uint64_t seed, uint64_t stream,
                     double sigma);

/* ------------------------------------------------------------ decode session
 * The whole-token device path: replaces the device branch of ForwardToken /
 * ForwardBatch (src/forward.cpp:292-333, :642-684) together with the greedy
 * GetArgMax of the sampler (src/ops.cpp:199-212, src/sampler.cpp:141-151).
 * One token = embedding, n_layers x (RMSNorm+QKV+bias, RoPE+KV write+split-K
 * attention, O-proj+residual, RMSNorm+gate/up+SwiGLU, down+residual), final
 * RMSNorm, lm_head, argmax, captured once as a CUDA graph whose position and
 * token live in device memory. */
typedef struct {
    int vocab_size;
    int dim;
    int hidden_dim;
    int n_layers;
    int n_heads;
    int n_kv_heads;
    int head_dim;
    int max_seq_len;
    float rope_theta;
    float rms_norm_eps;
    int rope_type;   /* mlb_rope_type */
    int weight_type; /* mlb_qtype of every linear weight (lm_head included) */
    int qkv_bias;    /* 1 when bq/bk/bv are present (Qwen2) */
} mlb_model_config; /* mirrors ModelConfig, include/model.h:16-28 */

typedef enum {
    MLB_W_EMBEDDING = 0, /* [vocab, dim] f32 */
    MLB_W_FINAL_NORM = 1,
    MLB_W_LM_HEAD = 2, /* [vocab, dim] weight_type */
    MLB_W_ATTN_NORM = 3,
    MLB_W_WQ = 4,
    MLB_W_WK = 5,
    MLB_W_WV = 6,
    MLB_W_BQ = 7,
    MLB_W_BK = 8,
    MLB_W_BV = 9,
    MLB_W_WO = 10,
    MLB_W_FFN_NORM = 11,
    MLB_W_GATE = 12,
    MLB_W_UP = 13,
    MLB_W_DOWN = 14
} mlb_weight_kind; /* the weight names of UploadModelWeightsToCuda, src/model.cpp:255-286 */

typedef struct mlb_model mlb_model;
typedef struct mlb_session mlb_session;

int mlb_model_create(int device, const mlb_model_config* config, mlb_model** model);
int mlb_model_destroy(mlb_model* model);
/* Device storage of one weight (allocated by the model); bytes is its size. */
int mlb_model_weight(mlb_model* model, int layer, int kind, void** dev_ptr, size_t* bytes);
/* Copies a weight from host (src_is_host = 1) or device memory. */
int mlb_model_set_weight(mlb_model* model, int layer, int kind, const void* src, size_t bytes,
                         int src_is_host);
/* Total bytes of device weight storage. */
int mlb_model_bytes(mlb_model* model, size_t* bytes);

int mlb_session_create(mlb_model* model, mlb_session** session);
int mlb_session_destroy(mlb_session* session);
/* Clears the KV cache (CudaKVCache::Clear, src/cuda_kv_cache.cpp:39-51). */
int mlb_session_reset(mlb_session* session);
/* ForwardToken: one token at position pos.  logits (host, vocab floats) and
 * next_token (host) may each be NULL. */
int mlb_session_forward(mlb_session* session, int token, int pos, float* logits,
                        int* next_token);
/* Greedy generation: forwards the prompt (host ids) at positions
 * start_pos.., then n_new greedy tokens (host out_tokens[n_new]); tokens are
 * fed back on the device. */
int mlb_session_generate(mlb_session* session, const int* prompt, int n_prompt, int start_pos,
                         int n_new, int* out_tokens);
/* Device-resident greedy decode for measurement: tokens (device int array of
 * n_steps + 1) holds the start token in tokens[0]; step i forwards tokens[i]
 * at position start_pos + i and writes the argmax to tokens[i + 1].  Enqueued
 * only; no host synchronisation. */
int mlb_session_decode_device(mlb_session* session, int* tokens, int start_pos, int n_steps);
/* Device pointer of the last logits (vocab floats). */
int mlb_session_logits(mlb_session* session, const float** logits);
/* Which decode path the session uses: 2 = the persistent decode kernel (one
 * cooperative launch per generate / decode_device / forward call, integer
 * tensor-core products over R16 weights), 1 = a CUDA graph per token whose
 * GEMVs are the integer tensor-core GEMV over R16 weights, 0 = a CUDA graph
 * per token with the bulk-copy SIMT GEMV over the GGUF blocks.  Q8_0 models
 * whose shapes fit get 2, other Q8_0 models 1, Q4_0 / Q4_1 models 0. */
int mlb_session_gemv_path(mlb_session* session, int* path);
/* Selects (enable = 1) or leaves (enable = 0) the persistent decode kernel
 * for this session; MLB_ERR_UNSUPPORTED when the model does not fit it.  No
 * reference counterpart: the per-token graph stays available for
 * comparison. */
int mlb_session_use_persistent(mlb_session* session, int enable);
/* Phase timeline of the persistent decode kernel (a profiling aid; no
 * reference counterpart).  With a device buffer of `entries` uint64, later
 * launches stamp %globaltimer (ns) at
 *   buffer[((step * (n_layers + 1) + layer) * 16 + event) * sm_count + cta]
 * for each CTA that takes part in the phase.  QKV: 0 wait done, 11 input
 * normalised, 10 products stored, 1 signalled.  Attention: 2 wait done,
 * 8 softmax.V done, 9 O-projection flushed, 3 signalled.  FFN: 4 wait done,
 * 7 input normalised, 6 down-projection flushed, 5 signalled.  Layer n_layers
 * (lm_head): 0 wait done, 1 done.  Stamps past `entries` are dropped; the
 * buffer is not cleared.  NULL, 0 turns the timeline off. */
int mlb_session_trace(mlb_session* session, unsigned long long* device_buffer, size_t entries);
/* Bound, in nanoseconds, of every wait inside the persistent decode kernel (a
 * dependency counter, a tagged hand-over word, a weight stage); default 2 s.
 * A wait that expires makes the call return MLB_ERR_DEVICE_TIMEOUT and leaves
 * the device usable.  No reference counterpart (the reference has no device
 * waits). */
int mlb_session_wait_limit(mlb_session* session, unsigned long long nanoseconds);
/* Test hook: the persistent kernel withholds every signal of phase counter
 * `counter` (layer l: 3l + 0 x_mid ready, 3l + 1 attention done, 3l + 2 FFN
 * done; -1 restores normal operation), so the waits on it expire after the
 * wait limit.  Exercises the bounded waits and the abort path without any
 * device fault.  No reference counterpart. */
int mlb_session_test_withhold_signal(mlb_session* session, int counter);
/* Device pointers of the session KV cache. */
int mlb_session_kv_cache(mlb_session* session, float** key_cache, float** value_cache);
/* Prompts of at least min_tokens tokens (default 16; 0: never) go through
 * mlb_session_generate in one pass -- every layer on all prompt tokens at
 * once, each linear one call on n_prompt rows (tensor cores from 9 rows),
 * RoPE and the KV write for all positions, then causal attention as a batch
 * of queries over the cache -- instead of one decode step per token.  The
 * per-position computation is the same; the reference processes prompts one
 * token at a time (ForwardBatch, src/forward.cpp:668-684). */
int mlb_session_prefill_min(mlb_session* session, int min_tokens);

/* ------------------------------------------------------------ batched decode
 * A batch of independent sequences decoded in lockstep through one model:
 * every step feeds one token per sequence (prompt tokens first, then the
 * greedy choice), so each linear runs on `batch` rows (the GEMV up to 8 rows,
 * the tensor cores from 9) and attention runs batched.  No reference
 * counterpart: the reference decodes one sequence at a time (ForwardBatch,
 * src/forward.cpp:668-684, loops ForwardToken); per sequence the computation
 * is that of mlb_session_generate, so the greedy tokens match it.
 *
 * Tensor parallelism: tp_size processes, one GPU each, build the same model
 * and each create a batch with its tp_rank and the same NCCL id (from
 * mlb_nccl_unique_id on one rank, shared by the caller).  Every linear's
 * output rows are split into tp_size contiguous slices -- q/k/v by KV-head
 * group, so each rank attends with its own KV heads and holds only their
 * cache -- and the slices are all-gathered with NCCL before the next step that
 * needs whole rows; the lm_head is split by vocabulary and the per-rank
 * arg-maxes are merged (first maximum wins).  tp_size must divide n_kv_heads,
 * dim, hidden_dim and vocab_size.  One step (all layers and the collectives)
 * is captured once as a CUDA graph. */
typedef struct mlb_batch mlb_batch;
#define MLB_NCCL_ID_BYTES 128
/* An NCCL unique id (MLB_NCCL_ID_BYTES bytes) for one tensor-parallel group. */
int mlb_nccl_unique_id(void* id);
/* The slices rank tp_rank owns, as 5 half-open ranges (10 ints): query heads,
 * KV heads, dim rows (wo, w_down), hidden rows (w_gate, w_up), vocabulary
 * rows (lm_head).  MLB_ERR_UNSUPPORTED when tp_size does not divide them. */
int mlb_batch_shard(const mlb_model_config* config, int tp_rank, int tp_size, int* ranges);
/* nccl_id may be NULL when tp_size == 1. */
int mlb_batch_create(mlb_model* model, int batch, int tp_rank, int tp_size, const void* nccl_id,
                     mlb_batch** out);
int mlb_batch_destroy(mlb_batch* batch);
/* Greedy continuation of `batch` prompts of n_prompt tokens each (host
 * [batch][n_prompt]) by n_new tokens (host out_tokens [batch][n_new]), from
 * position 0.  prefill_ms / decode_ms (may be NULL) receive the device time of
 * the n_prompt prompt steps and of the n_new - 1 further steps. */
int mlb_batch_generate(mlb_batch* batch, const int* prompts, int n_prompt, int n_new, int* out_tokens,
                       float* prefill_ms, float* decode_ms);
/* Device pointer of the last step's logits slice ([batch][cols], this rank's
 * vocabulary rows col0 .. col0 + cols - 1). */
int mlb_batch_logits(mlb_batch* batch, const float** logits, int* cols, int* col0);

#ifdef __cplusplus
}
#endif
#endif
