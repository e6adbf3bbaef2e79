// Persistent decode kernel: every decode step of a Q8_0 model (embedding,
// n_layers x transformer layer, final RMSNorm, lm_head, greedy arg-max) in one
// cooperative launch, for n_steps tokens in a row.
//
// Grid: one CTA per SM, all co-resident (cooperative launch), eight warps a
// CTA.  The work of a step is a fixed schedule of items per CTA:
//   QKV(l)   16-row tiles of [wq; wk; wv]          input x      -> qkv (+bias)
//   ATTO(l)  one query head: RoPE, KV write, attention over 0..pos, then the
//            head's 64 outputs times its block columns of wo, accumulated into
//            x_mid with red.add (x_mid starts as x)
//   FFN(l)   per 32-unit hidden block: its 32 gate and 32 up rows, SwiGLU,
//            then its w_down block column; the CTA sums its columns in shared
//            memory and adds them into the next x with one red.add pass (x
//            starts at zero; CTA 0 adds x_mid)
//   LM       16-row tiles of lm_head -> logits; per-CTA arg-max; the last CTA
//            to finish picks the token and releases the next step
// QKV hands q, k, v to the attention CTAs as tagged 64-bit words (value and
// the step's layer tag in one single-copy-atomic store) that the readers poll
// directly; the other phases (kMkPhases a layer) are ordered by global counters (release by an atomic add after a
// fence, acquire by polling).  Weights never depend on data, so each CTA
// streams its whole schedule (bulk copies into a ring of mbarrier-guarded
// stages) as far ahead as the ring allows, across phases and steps: thread 0
// refills a stage with the chunk kMkStages further on as soon as the CTA has
// released it.  (Without a separate copy warp each thread may hold up to 255
// registers; with nine warps an SM sub-partition would cap it at 168.)
//
// All weights are in the R16 layout (row tiles, qmma.cuh); wo and w_down in
// its column-major variant R16C so a block column is one contiguous copy.  Products are
// the exact integer block sums of qmma.cuh (mma.m16n8k32.s8 on int8 digit
// planes of the activations).
//
// Every wait is bounded: a wait that expires, or sees another CTA's abort,
// sets the status word and the CTA leaves its step loop; thread 0 then
// drains the copies still in flight before the CTA exits.
#pragma once

#include <string>

#include "qmma.cuh"

namespace mlb {

constexpr int kMkConsumerWarps = 8;
constexpr int kMkThreads = kMkConsumerWarps * 32;
constexpr int kMkStages = 4;
constexpr int kMkPhases = 3;        // counters per layer: QKV, attention, FFN
constexpr int kMkAttnChunk = 256;   // positions per attention pass (one per consumer thread)
constexpr int kMkTraceEvents = 16;  // timeline stamps per (step, layer, CTA)

struct MegaLayer {
    const uint8_t* wqkv[3];  // R16 wq, wk, wv
    const float* bias[3];    // bq, bk, bv (may be null)
    const float* attn_norm;
    const float* ffn_norm;
    const uint8_t* wo;    // R16C [dim, qd]
    const uint8_t* gate;  // R16 [hidden, dim]
    const uint8_t* up;    // R16 [hidden, dim]
    const uint8_t* down;  // R16C [dim, hidden]
};

struct MegaParams {
    int n_layers, dim, hidden, vocab, n_heads, n_kv, hd, max_seq, qd, kd;
    int group;
    float eps, scale;
    int neox;
    const float* embedding;
    const float* final_norm;
    const uint8_t* lm_head;  // R16
    const MegaLayer* layers;
    const float* rope_cos;
    const float* rope_sin;
    float* kc;
    float* vc;
    float* xbuf[2];
    float* xmid;
    unsigned long long* qkvt;  // [qd + 2 kd] tagged q, k, v words (QKV -> attention)
    unsigned tag_base;         // tag of (step 0, layer 0); (step, l) -> tag_base + step * n_layers + l
    float* logits;
    float* am_val;
    int* am_idx;
    unsigned* counters;  // [kMkPhases * n_layers + 2] zeroed before the launch
    int* hist;           // token history [max_seq + 1]
    int start_pos;
    int n_steps;
    int gen_from;  // hist[pos + 1] is written only when pos + 1 >= gen_from
    int* next_token;
    int* status;
    unsigned long long wait_ns;  // bound of one wait (dependency counter, tagged word, weight stage)
    int withhold;                // test hook: this counter is never signalled (-1: none)
    int stage_bytes;
    int list_cap;  // capacity of the per-CTA chunk list (MegaListCap)
    int kst_rows;  // cached K rows an attention item stages in shared memory (0..kMkAttnChunk)
    // optional timeline: [step][layer 0..n_layers][event][CTA] %globaltimer
    // stamps; null when off.  Events: QKV 0 wait done, 11 input normalised,
    // 10 products stored, 1 signalled; attention 2 wait done, 8 softmax.V
    // done, 9 O-projection flushed, 3 signalled; FFN 4 wait done, 7 input
    // normalised, 6 down-projection flushed, 5 signalled; layer n_layers
    // (lm_head) 0 wait done, 1 ticket taken.
    unsigned long long* trace;
    size_t trace_cap;
};

// Upper bound of the chunks one CTA of a grid of G streams per step.
int MegaListCap(const MegaParams& p, int G);
// Dynamic shared memory of the kernel (depends on dim, stage_bytes, list_cap).
size_t MegaSmemBytes(const MegaParams& p);
// Raises the kernel's shared-memory limit to smem; empty when one CTA of it
// fits on every one of the sm_count SMs (a cooperative grid), else the reason.
std::string MegaFits(const MegaParams& p, size_t smem, int sm_count);
// One cooperative launch of sm_count CTAs (MegaFits must have returned true).
void LaunchMegaDecode(const MegaParams& p, int sm_count, size_t smem, cudaStream_t stream);

}  // namespace mlb
