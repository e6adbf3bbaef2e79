// The model object of the C ABI (mlb_model): every weight of a mini_llama
// ModelConfig (include/model.h:16-28) in one device arena, in the GGUF block
// layout the reference uploads (src/model.cpp:255-286), plus the R16 / R16C
// copies of Q8_0 linears used by the decode session.  Shared by the decode
// session (decode.cu) and the batched decode driver (batch.cu).
#pragma once

#include <array>
#include <string>
#include <vector>

#include "../../include/mlb.h"

struct mlb_model {
    int device = 0;
    mlb_model_config cfg = {};
    void* arena = nullptr;
    size_t arena_bytes = 0;
    struct Slot {
        size_t offset = 0;
        size_t bytes = 0;
    };
    Slot global[3];                        // embedding, final_norm, lm_head
    std::vector<std::array<Slot, 15>> layer;  // per layer, kinds 3..14
    float* rope_cos = nullptr;
    float* rope_sin = nullptr;
    // Q8_0 models: every linear weight also in the R16 layout (integer-MMA GEMV)
    void* r16 = nullptr;
    size_t r16_bytes = 0;
    Slot r16_lm_head;
    std::vector<std::array<Slot, 15>> r16_layer;
    // wo and w_down also in R16C (block columns contiguous) when the
    // persistent decode kernel can run the model
    bool r16c = false;
    std::string mega_reason = "weights are not Q8_0";  // why not, when r16c is false
    std::vector<std::array<Slot, 2>> r16c_layer;

    void* Ptr(const Slot& s) const { return s.bytes ? static_cast<char*>(arena) + s.offset : nullptr; }
    const Slot& Get(int l, int kind) const {
        return kind < 3 ? global[kind] : layer[l][kind];
    }
    const uint8_t* R16(int l, int kind) const {
        const Slot& s = kind == MLB_W_LM_HEAD ? r16_lm_head : r16_layer[l][kind];
        return static_cast<const uint8_t*>(r16) + s.offset;
    }
    const uint8_t* R16C(int l, int kind) const {
        return static_cast<const uint8_t*>(r16) + r16c_layer[l][kind == MLB_W_WO ? 0 : 1].offset;
    }
};

