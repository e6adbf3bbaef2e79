// Host side of the integer-MMA Q8_0 GEMV over R16 weights: planning, launches
// and the C-ABI entry points that expose the prepared-weight form.
#include <algorithm>

#include "qmma.cuh"

namespace mlb {

GemvPlan PlanQmma(GemvParams& p, int M, bool dual, int sm_count, int max_smem, int ctas_per_sm,
                  int ring_budget) {
    GemvPlan plan;
    p.nb = (p.K + 31) / 32;
    p.rowbytes = p.nb * 34;
    p.M = M;
    const int nseg = dual ? 2 : p.nseg;
    for (int s = 0; s < nseg; ++s) {
        if (reinterpret_cast<uintptr_t>(p.seg[s].w) & 15) return plan;
        p.seg[s].tile_rows = 16;
        p.seg[s].tiles = (p.seg[s].rows + 15) / 16;
    }
    int total = 0;
    for (int s = 0; s < (dual ? 1 : p.nseg); ++s) total += p.seg[s].tiles;
    p.total_tiles = total;
    const long long tile_bytes = 1LL * p.nb * kR16Chunk;
    p.stage_bytes = static_cast<int>(tile_bytes * (dual ? 2 : 1));
    p.aux_floats = 0;
    if (p.norm_w) p.aux_floats = p.K;
    if (p.part_ml) p.aux_floats = p.n_heads * p.chunks * (p.head_dim + 2);
    int nst = std::max(2, std::min(4, ring_budget / std::max(1, p.stage_bytes)));
    for (; nst >= 2; --nst) {
        plan.smem = QmmaSmem::Bytes(M, p.nb, p.stage_bytes, nst, p.aux_floats);
        if (plan.smem + 4096 <= static_cast<size_t>(max_smem)) break;
    }
    if (nst < 2) return plan;
    p.nstages = nst;
    plan.grid = std::max(1, std::min(total, sm_count * ctas_per_sm));
    plan.ok = true;
    return plan;
}

template <int M, int PRO, int EPI>
void LaunchQmmaT(const GemvParams& p, const GemvPlan& plan, cudaStream_t stream, bool pdl) {
    auto kernel = QmmaGemvKernel<M, PRO, EPI>;
    static int configured[64] = {};
    int dev = 0;
    CheckCuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev >= 64 || configured[dev] < static_cast<int>(plan.smem)) {
        CheckCuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(plan.smem)),
                  "cudaFuncSetAttribute(QmmaGemvKernel)");
        if (dev < 64) configured[dev] = static_cast<int>(plan.smem);
    }
    Launch("QmmaGemvKernel", kernel, dim3(plan.grid), dim3(256), plan.smem, stream, pdl, p);
}

void LaunchQmmaDecode(int pro, int epi, const GemvParams& p, const GemvPlan& plan,
                      cudaStream_t stream) {
    if (pro == kProRmsNorm && epi == kEpiStore)
        return LaunchQmmaT<1, kProRmsNorm, kEpiStore>(p, plan, stream, true);
    if (pro == kProPlain && epi == kEpiResidual)
        return LaunchQmmaT<1, kProPlain, kEpiResidual>(p, plan, stream, true);
    if (pro == kProAttnMerge && epi == kEpiResidual)
        return LaunchQmmaT<1, kProAttnMerge, kEpiResidual>(p, plan, stream, true);
    if (pro == kProRmsNorm && epi == kEpiSwiglu)
        return LaunchQmmaT<1, kProRmsNorm, kEpiSwiglu>(p, plan, stream, true);
    if (pro == kProRmsNorm && epi == kEpiArgmax)
        return LaunchQmmaT<1, kProRmsNorm, kEpiArgmax>(p, plan, stream, true);
    Fail(MLB_ERR_UNSUPPORTED, "integer-MMA GEMV variant not built");
}

void LaunchQmmaStore(const GemvParams& p, const GemvPlan& plan, cudaStream_t stream) {
    switch (p.M) {
        case 1: return LaunchQmmaT<1, kProPlain, kEpiStore>(p, plan, stream, false);
        case 2: return LaunchQmmaT<2, kProPlain, kEpiStore>(p, plan, stream, false);
        case 3: return LaunchQmmaT<3, kProPlain, kEpiStore>(p, plan, stream, false);
        case 4: return LaunchQmmaT<4, kProPlain, kEpiStore>(p, plan, stream, false);
        case 5: return LaunchQmmaT<5, kProPlain, kEpiStore>(p, plan, stream, false);
        case 6: return LaunchQmmaT<6, kProPlain, kEpiStore>(p, plan, stream, false);
        case 7: return LaunchQmmaT<7, kProPlain, kEpiStore>(p, plan, stream, false);
        case 8: return LaunchQmmaT<8, kProPlain, kEpiStore>(p, plan, stream, false);
    }
    Fail(MLB_ERR_UNSUPPORTED, "integer-MMA GEMV: unsupported row count");
}

void LaunchRepackQ80R16(DeviceContext& c, const void* src, int rows, int cols, void* dst,
                        bool column_major) {
    const long long items = (rows + 15) / 16 * 16LL * ((cols + 31) / 32);
    const long long blocks = std::min<long long>((items + 255) / 256, 8LL * c.sm_count);
    RepackQ80R16Kernel<<<static_cast<unsigned>(std::max<long long>(blocks, 1)), 256, 0, c.stream>>>(
        static_cast<const uint8_t*>(src), rows, cols, static_cast<uint8_t*>(dst),
        column_major ? 1 : 0);
    CheckCuda(cudaGetLastError(), "RepackQ80R16Kernel");
}

}  // namespace mlb

using namespace mlb;

extern "C" {

size_t mlb_r16_bytes(int rows, int cols) {
    if (rows <= 0 || cols <= 0) return 0;
    return R16Bytes(rows, cols);
}

int mlb_q80_repack_r16(int device, const void* w, int rows, int cols, void* w_r16) {
    return Guard([&] {
        const char* c = "mlb_q80_repack_r16";
        Require(w && w_r16, c, "weight pointer is null");
        Require(rows > 0 && cols > 0, c, "dimension must be positive");
        LaunchRepackQ80R16(Ctx(device), w, rows, cols, w_r16);
    });
}

int mlb_q80_linear_r16(int device, const float* x, const void* w_r16, int rows, int in_features,
                       int out_features, const float* bias, float* y) {
    return Guard([&] {
        const char* c = "mlb_q80_linear_r16";
        Require(x && w_r16 && y, c, "input, weight or output pointer is null");
        Require(rows > 0 && in_features > 0 && out_features > 0, c,
                "empty tensors are not supported");
        Require((reinterpret_cast<uintptr_t>(w_r16) & 15) == 0, c,
                "R16 weights must be 16-byte aligned");
        DeviceContext& ctx = Ctx(device);
        for (int m0 = 0; m0 < rows;) {
            int M = std::min(rows - m0, kGemvMaxM);
            GemvParams p = {};
            GemvPlan plan;
            for (;;) {
                p = GemvParams{};
                p.K = in_features;
                p.nseg = 1;
                p.seg[0] = GemvSeg{static_cast<const uint8_t*>(w_r16), bias, out_features, 0, 0, 0};
                p.y_stride = out_features;
                plan = PlanQmma(p, M, false, ctx.sm_count, ctx.max_smem_optin, 1, 160 * 1024);
                if (plan.ok || M == 1) break;
                M = (M + 1) / 2;
            }
            Require(plan.ok, c, "shape does not fit shared memory", MLB_ERR_UNSUPPORTED);
            p.x = x + size_t(m0) * in_features;
            p.y = y + size_t(m0) * out_features;
            LaunchQmmaStore(p, plan, ctx.stream);
            m0 += M;
        }
    });
}

}  // extern "C"
