/*
 * CPU oracle for the mini_llama decode/prefill hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * CPU algorithms (mini_llama src/quant.cpp, src/ops.cpp, src/context.cpp,
 * src/forward.cpp, test/gpu_core_test.cpp), kept operation-for-operation in the
 * same fp32 order so that its outputs are bit-identical to the reference CPU
 * path built from source.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it, and only as the checker.
 *
 * Parity pin: tests/test_oracle_golden.py compares every function here with
 * golden vectors produced by the reference itself (oracle/_ref, built from the
 * reference sources by oracle/Makefile; fixtures in tests/golden/).
 */
#ifndef MLB_ORACLE_H
#define MLB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORC_F32 = 0, ORC_Q80 = 1, ORC_Q40 = 2, ORC_Q41 = 3 };

typedef struct {
    uint16_t d;
    int8_t qs[32];
} orc_block_q80; /* 34 bytes, mini_llama include/quantized_tensor.h:19-23 */

typedef struct {
    uint16_t d;
    uint8_t qs[16];
} orc_block_q40; /* 18 bytes, include/quantized_tensor.h:25-29 */

typedef struct {
    uint16_t d;
    uint16_t m;
    uint8_t qs[16];
} orc_block_q41; /* 20 bytes, include/quantized_tensor.h:32-37 */

uint16_t orc_f32_to_f16(float value);
float orc_f16_to_f32(uint16_t value);
size_t orc_block_bytes(int qtype);

/* x: rows x cols row-major; out: rows * ceil(cols/32) blocks. */
void orc_quantize(int qtype, const float* x, int rows, int cols, void* out);
void orc_dequantize(int qtype, const void* blocks, int rows, int cols, float* out);

/* y[M,N] = x[M,K] . dequant(W[N,K])^T, one sequential fp32 sum per output. */
void orc_linear(int qtype, const float* x, int M, int K, const void* w, int N, float* y,
                int threads);

void orc_rmsnorm(const float* x, const float* w, int n, float eps, float* y);
void orc_rope_tables(int max_seq_len, int head_dim, float theta, float* cos_t, float* sin_t);
void orc_rope_apply(float* x, int rows, int head_dim, int pos, const float* cos_t,
                    const float* sin_t, int neox);
/* Reference GPU-test RoPE (test/gpu_core_test.cpp:200-219): freq and angle
 * computed per call rather than from tables. */
void orc_rope_direct(float* x, int rows, int head_dim, int pos, float theta, int neox);
/* cache layout [n_layers, max_seq_len, n_kv_heads, head_dim] fp32.  scratch >= pos+1. */
void orc_attention(const float* q, const float* kcache, const float* vcache, int layer, int pos,
                   int max_seq_len, int n_heads, int n_kv_heads, int head_dim, float* out,
                   float* scratch);
void orc_softmax(const float* x, int n, float* y);
void orc_silu(const float* x, int n, float* y);
void orc_swiglu(const float* gate, const float* up, int n, float* y);
int orc_argmax(const float* x, int n);

/* ---- synthetic transformer ---- */
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
    int rope_neox;
    int qkv_bias;
    int tied_embedding;
    int qtype;
} orc_config;

enum {
    ORC_T_EMBEDDING = 0,
    ORC_T_FINAL_NORM = 1,
    ORC_T_LM_HEAD = 2,
    ORC_T_ATTN_NORM = 3,
    ORC_T_WQ = 4,
    ORC_T_WK = 5,
    ORC_T_WV = 6,
    ORC_T_BQ = 7,
    ORC_T_BK = 8,
    ORC_T_BV = 9,
    ORC_T_WO = 10,
    ORC_T_FFN_NORM = 11,
    ORC_T_GATE = 12,
    ORC_T_UP = 13,
    ORC_T_DOWN = 14,
};

typedef struct orc_model orc_model;

orc_model* orc_model_create_synth(const orc_config* cfg, uint64_t seed, int threads);
void orc_model_free(orc_model* m);
/* Pointer to a tensor's bytes (quantized blocks for linears, fp32 otherwise);
 * NULL when absent (e.g. biases without qkv_bias). */
const void* orc_model_tensor(const orc_model* m, int layer, int kind, size_t* bytes);
/* Clears the KV cache. */
void orc_model_reset(orc_model* m);
/* One token through all layers at position pos; writes vocab_size logits. */
int orc_model_forward(orc_model* m, int token, int pos, float* logits);

void orc_synth_normal(float* out, size_t n, uint64_t seed, uint64_t stream, double sigma,
                      int threads);
void orc_synth_tokens(int* out, int n, uint64_t seed, int vocab);

#ifdef __cplusplus
}
#endif
#endif
