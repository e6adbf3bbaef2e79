// Quantized linear entry points (replace mini_llama include/cuda_quant.h:13-38
// and the kernels of src/cuda_quant.cu:40-135).
#include <algorithm>
#include <numeric>

#include "blockmma.cuh"
#include "qgemv.cuh"

namespace mlb {

namespace {
int Gcd(int a, int b) { return b == 0 ? a : Gcd(b, a % b); }
}  // namespace

GemvPlan PlanGemv(GemvParams& p, int qtype, int M, bool dual, int sm_count, int max_smem,
                  int ctas_per_sm, int ring_budget) {
    GemvPlan plan;
    const int bb = BlockBytes(qtype);
    p.nb = (p.K + 31) / 32;
    p.rowbytes = p.nb * bb;
    p.M = M;
    const int nseg = dual ? 2 : p.nseg;
    for (int s = 0; s < nseg; ++s) {
        if (reinterpret_cast<uintptr_t>(p.seg[s].w) & 15) return plan;
    }
    const int rg = 16 / Gcd(p.rowbytes, 16);
    int part_cap = 16384;
    while (part_cap < rg * p.rowbytes && part_cap < 49152) part_cap += 16384;
    if (rg * p.rowbytes > part_cap) return plan;
    int r_cap = (part_cap / p.rowbytes) / rg * rg;
    r_cap = std::min(r_cap, kGemvMaxTileRows / rg * rg);
    const int r_ring = (ring_budget / (kGemvStages * p.rowbytes * (dual ? 2 : 1))) / rg * rg;
    if (r_ring >= rg) r_cap = std::min(r_cap, r_ring);
    long long total_rows = 0;
    for (int s = 0; s < (dual ? 1 : p.nseg); ++s) total_rows += p.seg[s].rows;
    const long long want_tiles = 2LL * sm_count * ctas_per_sm;
    int r_par = static_cast<int>((total_rows + want_tiles - 1) / want_tiles);
    r_par = (r_par + rg - 1) / rg * rg;
    const int R = std::max(rg, std::min(r_cap, r_par));
    int total = 0;
    for (int s = 0; s < nseg; ++s) {
        p.seg[s].tile_rows = R;
        p.seg[s].tiles = (p.seg[s].rows + R - 1) / R;
        if (!dual || s == 0) total += p.seg[s].tiles;
    }
    p.total_tiles = total;
    const int part_bytes = (R * p.rowbytes + 15) / 16 * 16;
    p.stage_bytes = dual ? 2 * part_bytes : part_bytes;
    p.aux_floats = 0;
    if (p.norm_w) p.aux_floats = p.K;
    if (p.part_ml) p.aux_floats = p.n_heads * p.chunks * (p.head_dim + 2);
    plan.smem = GemvSmem::Bytes(M, p.nb, p.stage_bytes, p.aux_floats);
    if (plan.smem + 4096 > static_cast<size_t>(max_smem)) return plan;
    // no more CTAs than fit on the SMs at once (an SM's shared memory is the
    // per-block maximum plus the 1 KB the runtime reserves per block): a
    // second wave would stage x again and start its ring late
    const int resident = std::max(1, static_cast<int>((static_cast<size_t>(max_smem) + 1024) / (plan.smem + 1024)));
    plan.grid = std::max(1, std::min(total, sm_count * std::min(ctas_per_sm, resident)));
    plan.ok = true;
    return plan;
}

BmPlan PlanBlockMma(BmParams& p, int qtype, int M, int sm_count, int max_smem) {
    BmPlan plan;
    const int bb = BlockBytes(qtype);
    p.nb = (p.K + 31) / 32;
    p.rowbytes = p.nb * bb;
    p.tiles = (p.N + 15) / 16;
    if (reinterpret_cast<uintptr_t>(p.w) & 15) return plan;
    // Q8_0 / Q4_0 blocks are read in pairs
    if (qtype != MLB_Q4_1 && (p.nb & 1)) return plan;
    constexpr int kMaxStage = 20 * 1024;
    const long long tile_bytes = 16LL * p.rowbytes;
    if (tile_bytes <= kMaxStage) {
        p.kc = p.nb;
        p.units_k = 1;
        p.pitch = p.rowbytes;  // 16 contiguous GGUF rows
        p.stage_bytes = static_cast<int>((tile_bytes + 15) & ~15LL);
    } else if (p.rowbytes % 16 == 0) {
        // pieces of kc blocks (a multiple of 8) start and end 16-byte aligned;
        // rows land at a pitch of 16 mod 32 bytes (4 mod 8 words)
        p.kc = std::min(p.nb, std::max(8, kMaxStage / (16 * bb) / 8 * 8));
        p.units_k = (p.nb + p.kc - 1) / p.kc;
        p.pitch = p.kc * bb;
        if (p.pitch % 32 == 0) p.pitch += 16;
        p.stage_bytes = 16 * p.pitch;
    } else {
        return plan;
    }
    // Too few row tiles to stream: the other GEMV (K split across warps)
    // finishes sooner below about 4 row tiles per SM (measured on whole rows
    // and on rows split into pieces, where a pair runs a tile's pieces one
    // after another).
    if (p.tiles < 4 * sm_count) return plan;
    p.rowmap = ((p.pitch / 4) % 4 == 2) ? 1 : 0;
    // Warp pairs with a two-slot ring each (groups of 4 warps with 3 or 4
    // slots, splitting each tile 4 ways, measured slower at every row count)
    p.gsize = kBmGroupWarps;
    p.slots = 2;
    const bool sums = qtype == MLB_Q4_1;
    const size_t budget = static_cast<size_t>(max_smem) - 1024;
    plan.grid = sm_count;
    // as many groups as fit (the tile scheduler balances them), at most one
    // per tile of an SM's share
    int groups = std::min(kBmMaxWarps / p.gsize, (p.tiles + plan.grid - 1) / plan.grid);
    while (groups > 0 && BmSmem::Bytes(M, p.nb, groups, p.slots, p.stage_bytes, sums, p.gsize) > budget) --groups;
    // x's tables span all of K: when they leave room for fewer than six
    // warps (long rows, many rows of x), too few copies are in flight
    if (groups * p.gsize < std::min(6, p.gsize * ((p.tiles + plan.grid - 1) / plan.grid))) return plan;
    plan.warps = groups * p.gsize;
    plan.smem = BmSmem::Bytes(M, p.nb, groups, p.slots, p.stage_bytes, sums, p.gsize);
    plan.ok = plan.smem <= budget;
    return plan;
}

template <int QT, int M>
void LaunchBlockMmaT(const BmParams& p, const BmPlan& plan, cudaStream_t stream) {
    auto kernel = BlockMmaGemvKernel<QT, M>;
    static int configured_smem[64] = {};  // per instantiation and device
    int dev = 0;
    CheckCuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev >= 64 || configured_smem[dev] < static_cast<int>(plan.smem)) {
        CheckCuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(plan.smem)),
                  "cudaFuncSetAttribute(BlockMmaGemvKernel)");
        if (dev < 64) configured_smem[dev] = static_cast<int>(plan.smem);
    }
    Launch("BlockMmaGemvKernel", kernel, dim3(plan.grid), dim3(32 * plan.warps), plan.smem, stream,
           false, p);
}

template <int QT>
void LaunchBlockMmaM(int M, const BmParams& p, const BmPlan& plan, cudaStream_t stream) {
    switch (M) {
        case 1: return LaunchBlockMmaT<QT, 1>(p, plan, stream);
        case 2: return LaunchBlockMmaT<QT, 2>(p, plan, stream);
        case 3: return LaunchBlockMmaT<QT, 3>(p, plan, stream);
        case 4: return LaunchBlockMmaT<QT, 4>(p, plan, stream);
        case 5: return LaunchBlockMmaT<QT, 5>(p, plan, stream);
        case 6: return LaunchBlockMmaT<QT, 6>(p, plan, stream);
        case 7: return LaunchBlockMmaT<QT, 7>(p, plan, stream);
        case 8: return LaunchBlockMmaT<QT, 8>(p, plan, stream);
    }
    Fail(MLB_ERR_UNSUPPORTED, "block-MMA GEMV: unsupported row count");
}

void LaunchBlockMma(int qtype, int M, const BmParams& p, const BmPlan& plan, cudaStream_t stream) {
    switch (qtype) {
        case MLB_Q8_0: return LaunchBlockMmaM<MLB_Q8_0>(M, p, plan, stream);
        case MLB_Q4_0: return LaunchBlockMmaM<MLB_Q4_0>(M, p, plan, stream);
        case MLB_Q4_1: return LaunchBlockMmaM<MLB_Q4_1>(M, p, plan, stream);
    }
    Fail(MLB_ERR_UNSUPPORTED, "block-MMA GEMV: unsupported block type");
}

template <int QT, int M, int PRO, int EPI>
void LaunchGemvT(const GemvParams& p, const GemvPlan& plan, cudaStream_t stream, bool pdl) {
    auto kernel = GemvKernel<QT, M, PRO, EPI>;
    static int configured_smem[64] = {};  // per instantiation and device
    int dev = 0;
    CheckCuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev >= 64 || configured_smem[dev] < static_cast<int>(plan.smem)) {
        CheckCuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(plan.smem)),
                  "cudaFuncSetAttribute(GemvKernel)");
        if (dev < 64) configured_smem[dev] = static_cast<int>(plan.smem);
    }
    Launch("GemvKernel", kernel, dim3(plan.grid), dim3(kGemvThreads), plan.smem, stream, pdl, p);
}

template <int QT, int PRO, int EPI>
void LaunchGemvM(const GemvParams& p, const GemvPlan& plan, cudaStream_t stream, bool pdl) {
    switch (p.M) {
        case 1: return LaunchGemvT<QT, 1, PRO, EPI>(p, plan, stream, pdl);
        case 2: return LaunchGemvT<QT, 2, PRO, EPI>(p, plan, stream, pdl);
        case 3: return LaunchGemvT<QT, 3, PRO, EPI>(p, plan, stream, pdl);
        case 4: return LaunchGemvT<QT, 4, PRO, EPI>(p, plan, stream, pdl);
        case 5: return LaunchGemvT<QT, 5, PRO, EPI>(p, plan, stream, pdl);
        case 6: return LaunchGemvT<QT, 6, PRO, EPI>(p, plan, stream, pdl);
        case 7: return LaunchGemvT<QT, 7, PRO, EPI>(p, plan, stream, pdl);
        case 8: return LaunchGemvT<QT, 8, PRO, EPI>(p, plan, stream, pdl);
    }
    Fail(MLB_ERR_UNSUPPORTED, "GEMV: unsupported row count");
}

void LaunchGemvDecode(int qtype, int pro, int epi, const GemvParams& p, const GemvPlan& plan,
                      cudaStream_t stream) {
    // M = 1 variants used by the decode graph (programmatic dependent launch on)
#define MLB_GEMV_CASE(QT)                                                                      \
    if (qtype == QT) {                                                                         \
        if (pro == kProRmsNorm && epi == kEpiStore)                                            \
            return LaunchGemvT<QT, 1, kProRmsNorm, kEpiStore>(p, plan, stream, true);          \
        if (pro == kProPlain && epi == kEpiResidual)                                           \
            return LaunchGemvT<QT, 1, kProPlain, kEpiResidual>(p, plan, stream, true);         \
        if (pro == kProAttnMerge && epi == kEpiResidual)                                       \
            return LaunchGemvT<QT, 1, kProAttnMerge, kEpiResidual>(p, plan, stream, true);     \
        if (pro == kProRmsNorm && epi == kEpiSwiglu)                                           \
            return LaunchGemvT<QT, 1, kProRmsNorm, kEpiSwiglu>(p, plan, stream, true);         \
        if (pro == kProRmsNorm && epi == kEpiArgmax)                                           \
            return LaunchGemvT<QT, 1, kProRmsNorm, kEpiArgmax>(p, plan, stream, true);         \
    }
    MLB_GEMV_CASE(MLB_Q8_0)
    MLB_GEMV_CASE(MLB_Q4_0)
    MLB_GEMV_CASE(MLB_Q4_1)
#undef MLB_GEMV_CASE
    Fail(MLB_ERR_UNSUPPORTED, "decode GEMV variant not built");
}

void LaunchGemvStore(int qtype, const GemvParams& p, const GemvPlan& plan, cudaStream_t stream) {
    switch (qtype) {
        case MLB_Q8_0: return LaunchGemvM<MLB_Q8_0, kProPlain, kEpiStore>(p, plan, stream, false);
        case MLB_Q4_0: return LaunchGemvM<MLB_Q4_0, kProPlain, kEpiStore>(p, plan, stream, false);
        case MLB_Q4_1: return LaunchGemvM<MLB_Q4_1, kProPlain, kEpiStore>(p, plan, stream, false);
    }
}

template <int QT>
void LaunchFallback(const float* x, const uint8_t* w, const float* bias, float* y, int M, int K,
                    int N, cudaStream_t stream) {
    const int nb = (K + 31) / 32;
    const long long warps = 1LL * N * M;
    const int threads = 256;
    const long long blocks = (warps * 32 + threads - 1) / threads;
    GemvFallbackKernel<QT><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(x, w, bias, y, M,
                                                                                   K, N, nb);
    CheckCuda(cudaGetLastError(), "GemvFallbackKernel");
}

// Shared by the entry points: validation with the reference's messages
// (src/cuda_quant.cu:184-210), then LinearRows.
void QuantLinear(const char* caller, int device, int qtype, const float* x, const void* w,
                 size_t block_count, int rows, int in_features, int out_features,
                 const float* bias, float* y) {
    Require(qtype == MLB_Q8_0 || qtype == MLB_Q4_0 || qtype == MLB_Q4_1, caller,
            "unsupported block type");
    Require(w != nullptr, caller, "device weight pointer is null");
    Require(x != nullptr && y != nullptr, caller, "input or output pointer is null");
    Require(rows > 0 && in_features > 0 && out_features > 0, caller,
            "empty tensors are not supported");
    const int nb = (in_features + 31) / 32;
    const size_t expected = static_cast<size_t>(out_features) * nb;
    Require(block_count == expected, caller,
            "block count mismatch: expected " + std::to_string(expected) + ", got " +
                std::to_string(block_count));
    DeviceContext& c = Ctx(device);
    LinearRows(c, qtype, x, static_cast<const uint8_t*>(w), rows, in_features, out_features, bias, y);
}

void LinearRows(DeviceContext& c, int qtype, const float* x, const uint8_t* wb, int rows, int in_features,
                int out_features, const float* bias, float* y, void* tc_workspace, bool reuse_x) {
    if (rows >= kTcMinRows) {  // prefill-sized batches: tcgen05 tensor cores
        LaunchTcLinear(c, qtype, x, wb, rows, in_features, out_features, bias, y, c.status, tc_workspace, reuse_x);
        return;
    }

    for (int m0 = 0; m0 < rows;) {
        int M = std::min(rows - m0, kGemvMaxM);
        {
            // tensor-core GEMV over the blocks, when the shape suits it
            // (x's tables grow with the rows of x: when they leave too
            // little room, fewer rows per launch)
            BmParams bp;
            BmPlan bplan;
            int mb = M;
            for (;; mb = (mb + 1) / 2) {
                bp = BmParams{};
                bp.w = wb;
                bp.K = in_features;
                bp.N = out_features;
                bplan = PlanBlockMma(bp, qtype, mb, c.sm_count, c.max_smem_optin);
                if (bplan.ok || mb == 1) break;
            }
            if (bplan.ok) {
                M = mb;
                bp.x = x + static_cast<size_t>(m0) * in_features;
                bp.y = y + static_cast<size_t>(m0) * out_features;
                bp.bias = bias;
                bp.status = c.status;
                LaunchBlockMma(qtype, M, bp, bplan, c.stream);
                m0 += M;
                continue;
            }
        }
        GemvParams p = {};
        p.K = in_features;
        p.nseg = 1;
        p.seg[0] = GemvSeg{wb, bias, out_features, 0, 0, 0};
        p.y_stride = out_features;
        GemvPlan plan;
        for (;;) {
            plan = PlanGemv(p, qtype, M, false, c.sm_count, c.max_smem_optin, 3);
            if (plan.ok || M == 1) break;
            M = (M + 1) / 2;
            p = GemvParams{};
            p.K = in_features;
            p.nseg = 1;
            p.seg[0] = GemvSeg{wb, bias, out_features, 0, 0, 0};
            p.y_stride = out_features;
        }
        const float* xm = x + static_cast<size_t>(m0) * in_features;
        float* ym = y + static_cast<size_t>(m0) * out_features;
        if (plan.ok) {
            p.x = xm;
            p.y = ym;
            LaunchGemvStore(qtype, p, plan, c.stream);
        } else {
            if (qtype == MLB_Q8_0) LaunchFallback<MLB_Q8_0>(xm, wb, bias, ym, M, in_features,
                                                            out_features, c.stream);
            else if (qtype == MLB_Q4_0) LaunchFallback<MLB_Q4_0>(xm, wb, bias, ym, M,
                                                                 in_features, out_features,
                                                                 c.stream);
            else LaunchFallback<MLB_Q4_1>(xm, wb, bias, ym, M, in_features, out_features,
                                          c.stream);
        }
        m0 += M;
    }
}

}  // namespace mlb

using namespace mlb;

extern "C" {

int mlb_quant_linear(int device, int qtype, const float* x, const void* w, size_t block_count,
                     int rows, int in_features, int out_features, const float* bias, float* y) {
    return Guard([&] {
        QuantLinear("mlb_quant_linear", device, qtype, x, w, block_count, rows, in_features,
                    out_features, bias, y);
    });
}

int mlb_q80_linear(int device, const float* x, const void* w, size_t block_count, int rows,
                   int in_features, int out_features, const float* bias, float* y) {
    return Guard([&] {
        QuantLinear("CudaQ80Linear", device, MLB_Q8_0, x, w, block_count, rows, in_features,
                    out_features, bias, y);
    });
}

int mlb_q40_linear(int device, const float* x, const void* w, size_t block_count, int rows,
                   int in_features, int out_features, const float* bias, float* y) {
    return Guard([&] {
        QuantLinear("CudaQ40Linear", device, MLB_Q4_0, x, w, block_count, rows, in_features,
                    out_features, bias, y);
    });
}

int mlb_q41_linear(int device, const float* x, const void* w, size_t block_count, int rows,
                   int in_features, int out_features, const float* bias, float* y) {
    return Guard([&] {
        QuantLinear("CudaQ41Linear", device, MLB_Q4_1, x, w, block_count, rows, in_features,
                    out_features, bias, y);
    });
}

}  // extern "C"
