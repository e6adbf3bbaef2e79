// The split-K decode-attention kernel (design notes in attention.cuh).
#pragma once

namespace mlb {

// Single-float cp.async copies of tile rows r0 .. r0 + n into one ring stage
// (head_dim not a multiple of 4, or unaligned caches); rows at stride hdp.
// The row of this token (skip_row) is left out: its values come from kn / vn.
// No commit.
__device__ __forceinline__ void AttnCopyTile(int hd, int hdp, float* ks, float* vs, const float* kbase,
                                             const float* vbase, size_t pstride, int r0, int n, int skip_row) {
    for (int i = threadIdx.x; i < n * hd; i += kAttnThreads) {
        const int r = i / hd, d = i - r * hd;
        if (r0 + r == skip_row) continue;
        const size_t src = size_t(r0 + r) * pstride + d;
        CpAsync4(ks + r * hdp + d, kbase + src);
        CpAsync4(vs + r * hdp + d, vbase + src);
    }
}

// The two tensor-map boxes (K and V rows row .. row + T of KV head kvh) of a
// tile into one ring stage, completing on its mbarrier; one thread.  Rows
// past the maps' end arrive as zeros and still count toward the bytes.
__device__ __forceinline__ void AttnTmaTile(const CUtensorMap* kmap, const CUtensorMap* vmap, float* ks, float* vs,
                                            uint64_t* bar, int kvh, int row, uint32_t bytes) {
    MbarExpectTx(bar, bytes);
    TmaLoad3D(ks, kmap, 0, kvh, row, bar);
    TmaLoad3D(vs, vmap, 0, kvh, row, bar);
}

// GM: query heads per CTA rounded up to a power of two (1..kAttnGmax).
// TMA: tiles as tensor-map boxes (kmap, vmap: [rows][n_kv][hd] views of the
// caches) instead of cp.async copies.
template <int GM, bool TMA>
__global__ void __launch_bounds__(kAttnThreads, 2)
    AttnSplitKernel(const AttnParams p, const __grid_constant__ CUtensorMap kmap,
                    const __grid_constant__ CUtensorMap vmap) {
    extern __shared__ __align__(128) uint8_t abytes[];
    const AttnGeom G = AttnGeometry(p.hd);
    const int hd = p.hd, hdp = G.hdp, lpr = G.lpr, T = G.T, tpp = G.tpp;
    const int stage_f = T * hdp;
    const size_t ring_f = size_t(2) * kAttnStages * stage_f, red_f = size_t(G.R) * GM * hdp;
    uint64_t* full = reinterpret_cast<uint64_t*>(abytes);                  // [kAttnStages] mbarriers
    volatile int* abortf = reinterpret_cast<volatile int*>(abytes + 64);  // a tile wait gave up
    float* asmem = reinterpret_cast<float*>(abytes + kAttnHeader);
    float* ks = asmem;                           // [kAttnStages][T][hdp]
    float* vs = ks + kAttnStages * stage_f;      // [kAttnStages][T][hdp]
    float* red = asmem;                          // after the loop: [R][GM][hdp]
    float* qs = asmem + (ring_f > red_f ? ring_f : red_f);  // [GM][hdp]
    float* kn = qs + GM * hdp;                   // [hdp] this token's rotated k
    float* vn = kn + hdp;                        // [hdp] and v
    float* sp = vn + hdp;                        // [GM][T] scores, then weights (zero past the tile's rows)
    float* hm = sp + GM * T;                     // [GM] running maximum
    float* hl = hm + GM;                         // [GM] running sum
    float* hc = hl + GM;                         // [GM] the tile's correction factor

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kvh = blockIdx.x / p.hgroups, hg = blockIdx.x % p.hgroups;
    const int chunk = blockIdx.y, b = blockIdx.z;
    const int h0 = kvh * p.group + hg * kAttnGmax;
    const int gcnt = min(kAttnGmax, p.group - hg * kAttnGmax);  // <= GM (launch choice)

    GridDepWait();
    GridDepLaunch();

    // A position outside the cache (possible only through a device array)
    // attends to nothing and yields zeros instead of reading out of bounds.
    const int pos_raw = p.pos_dev ? p.pos_dev[size_t(b) * p.pos_stride] : p.pos_host;
    const bool valid = pos_raw >= 0 && pos_raw < p.max_seq_len;
    const int pos = valid ? pos_raw : 0;
    const int npos = valid ? pos_raw + 1 : 0;
    const int clen = (npos + p.chunks - 1) / p.chunks;
    const int p0 = min(npos, chunk * clen), p1 = min(npos, p0 + clen);
    const int ntiles = (p1 - p0 + T - 1) / T;
    const bool own_new = p.fused_rope && valid && pos >= p0 && pos < p1;
    const int skip_row = own_new ? pos : -1;

    const size_t pstride = size_t(p.n_kv) * hd;
    float* kbase = p.kc + size_t(b) * p.seq_stride + size_t(p.layer) * p.max_seq_len * pstride +
                   size_t(kvh) * hd;
    float* vbase = p.vc + size_t(b) * p.seq_stride + size_t(p.layer) * p.max_seq_len * pstride +
                   size_t(kvh) * hd;
    const int row0 = (p.seq_stride ? b * p.seq_rows : 0) + p.layer * p.max_seq_len + p0;  // map row of p0
    const uint32_t tile_bytes = 2u * static_cast<uint32_t>(T * hd) * 4u;
    const float* qsrc = p.q + size_t(b) * p.q_batch_stride + size_t(h0) * hd;

    // ---- prologue: the stages' barriers, the padding columns (never copy
    // targets) at zero, q of the group, the first kAttnStages - 1 tiles
    if constexpr (TMA) {
        if (tid == 0) {
            for (int i = 0; i < kAttnStages; ++i) MbarInit(&full[i], 1);
            *abortf = 0;
            FenceMbarInit();
            for (int t = 0; t < kAttnStages - 1 && t < ntiles; ++t)
                AttnTmaTile(&kmap, &vmap, ks + t * stage_f, vs + t * stage_f, &full[t], kvh, row0 + t * T,
                            tile_bytes);
        }
    } else if (hdp > hd) {
        for (int i = tid; i < 2 * kAttnStages * T * (hdp - hd); i += kAttnThreads) {
            const int rr = i / (hdp - hd);
            ks[rr * hdp + hd + (i - rr * (hdp - hd))] = 0.0f;  // K then V rows (vs follows ks)
        }
    }
    if (hdp > hd) {
        for (int i = tid; i < GM * (hdp - hd); i += kAttnThreads)
            qs[(i / (hdp - hd)) * hdp + hd + i % (hdp - hd)] = 0.0f;
        if (tid < hdp - hd) kn[hd + tid] = vn[hd + tid] = 0.0f;
    }
    const bool qvec = (hd & 3) == 0 && (reinterpret_cast<uintptr_t>(qsrc) & 15) == 0;
    if (qvec) {
        for (int i = tid; i < gcnt * lpr; i += kAttnThreads) {
            const int g = i / lpr, c = i - g * lpr;
            CpAsync16(qs + g * hdp + 4 * c, qsrc + size_t(g) * hd + 4 * c);
        }
    } else {
        for (int i = tid; i < gcnt * hd; i += kAttnThreads) {
            const int g = i / hd, d = i - g * hd;
            CpAsync4(qs + g * hdp + d, qsrc + size_t(g) * hd + d);
        }
    }
    CpAsyncCommit();
    if constexpr (!TMA) {
#pragma unroll
        for (int t = 0; t < kAttnStages - 1; ++t) {
            if (t < ntiles)
                AttnCopyTile(hd, hdp, ks + t * stage_f, vs + t * stage_f, kbase, vbase, pstride, p0 + t * T,
                             min(T, p1 - p0 - t * T), skip_row);
            CpAsyncCommit();
        }
    }
    if (tid < GM) {
        hm[tid] = -INFINITY;
        hl[tid] = 0.0f;
    }
    CpAsyncWaitGroup<TMA ? 0 : kAttnStages - 1>();  // this thread's q copies have landed
    __syncthreads();
    if (p.fused_rope && valid) {
        // RoPE with the reference CPU tables; the chunk holding `pos` also
        // rotates this token's k and stores k, v into the cache.
        const int half = hd / 2;
        const float* ct = p.rope_cos + size_t(pos) * half;
        const float* st = p.rope_sin + size_t(pos) * half;
        for (int i = tid; i < gcnt * half; i += kAttnThreads) {
            const int g = i / half, j = i - g * half;
            const int a = p.neox ? j : 2 * j, c2 = p.neox ? j + half : 2 * j + 1;
            const float x0 = qs[g * hdp + a], x1 = qs[g * hdp + c2], cs = ct[j], sn = st[j];
            qs[g * hdp + a] = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            qs[g * hdp + c2] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        }
        if (own_new) {
            const float* knew = p.kv_new + size_t(b) * p.kv_batch_stride + size_t(kvh) * hd;
            const float* vnew = (p.v_new ? p.v_new + size_t(b) * p.kv_batch_stride
                                         : p.kv_new + size_t(b) * p.kv_batch_stride + size_t(p.n_kv) * hd) +
                                size_t(kvh) * hd;
            float* kd = kbase + size_t(pos) * pstride;
            float* vd = vbase + size_t(pos) * pstride;
            for (int j = tid; j < half; j += kAttnThreads) {
                const int a = p.neox ? j : 2 * j, c2 = p.neox ? j + half : 2 * j + 1;
                const float x0 = knew[a], x1 = knew[c2], cs = ct[j], sn = st[j];
                const float ka = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
                const float kb = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
                kd[a] = ka;
                kd[c2] = kb;
                kn[a] = ka;
                kn[c2] = kb;
            }
            if ((hd & 1) && tid == 0) kd[hd - 1] = kn[hd - 1] = knew[hd - 1];  // no pair: unrotated
            for (int d = tid; d < hd; d += kAttnThreads) {
                const float v = vnew[d];
                vd[d] = v;
                vn[d] = v;
            }
        }
        __syncthreads();
    }

    // ---- tiles: scores, online softmax, weighted values
    float4 acc[GM];
#pragma unroll
    for (int g = 0; g < GM; ++g) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int sr = tid / tpp, ssub = tid - sr * tpp;  // score thread: row sr, pieces ssub + tpp i
    const int sperm = (((sr >> G.ksh) & G.kmk) * G.kml) / tpp;  // its piece order: i ^ sperm
    const int vrg = tid / lpr, vcol = tid - vrg * lpr;           // value thread: row group vrg, column vcol
    const bool vquad = T == 4 * G.R;  // rows 4 vrg .. 4 vrg + 3 per value thread (power-of-two rows)
    int t = 0;
    for (; t < ntiles; ++t) {
        const int st = t % kAttnStages;
        if constexpr (TMA) {
            if (!MbarWaitFor(&full[st], (t / kAttnStages) & 1, kAttnWaitNs, abortf)) {
                if (p.status) atomicCAS(p.status, 0, MLB_ERR_DEVICE_TIMEOUT);
                *abortf = 1;
            }
        } else {
            CpAsyncWaitGroup<kAttnStages - 2>();
        }
        __syncthreads();  // tile t has landed; every thread is done with tile t - 1 and its stage
        if constexpr (TMA) {
            if (*abortf) break;
        }
        {
            const int tn = t + kAttnStages - 1, sn = tn % kAttnStages;
            if constexpr (TMA) {
                if (tid == 0 && tn < ntiles)
                    AttnTmaTile(&kmap, &vmap, ks + sn * stage_f, vs + sn * stage_f, &full[sn], kvh, row0 + tn * T,
                                tile_bytes);
            } else {
                if (tn < ntiles)
                    AttnCopyTile(hd, hdp, ks + sn * stage_f, vs + sn * stage_f, kbase, vbase, pstride, p0 + tn * T,
                                 min(T, p1 - p0 - tn * T), skip_row);
                CpAsyncCommit();
            }
        }
        const int r0 = p0 + t * T, n = min(T, p1 - r0);
        const float* kt = ks + st * stage_f;
        const float* vt = vs + st * stage_f;
        {
            // rows past n hold stale data: their dots are formed (the
            // shuffles need every lane) and dropped
            float dot[GM];
#pragma unroll
            for (int g = 0; g < GM; ++g) dot[g] = 0.0f;
            const float* krow = r0 + sr == skip_row ? kn : kt + sr * hdp;
#pragma unroll 2
            for (int i = 0; i < kAttnPieces; ++i) {
                const int c = ssub + tpp * (i ^ sperm);
                if (c < lpr) {
                    const float4 kv = Lds4(krow + 4 * c);
#pragma unroll
                    for (int g = 0; g < GM; ++g)
                        if (g < gcnt) {
                            const float4 qv = Lds4(qs + g * hdp + 4 * c);
                            dot[g] = fmaf(qv.x, kv.x, dot[g]);
                            dot[g] = fmaf(qv.y, kv.y, dot[g]);
                            dot[g] = fmaf(qv.z, kv.z, dot[g]);
                            dot[g] = fmaf(qv.w, kv.w, dot[g]);
                        }
                }
            }
            for (int o = 1; o < tpp; o <<= 1)
#pragma unroll
                for (int g = 0; g < GM; ++g) dot[g] += __shfl_xor_sync(0xffffffffu, dot[g], o);
            if (ssub == 0 && sr < n)
#pragma unroll
                for (int g = 0; g < GM; ++g)
                    if (g < gcnt) sp[g * T + sr] = dot[g] * p.scale;
        }
        __syncthreads();
        for (int g = warp; g < gcnt; g += kAttnWarps) {  // softmax of the tile, a warp per head
            float mt = -INFINITY;
            for (int r = lane; r < n; r += 32) mt = fmaxf(mt, sp[g * T + r]);
            mt = WarpMax(mt);
            const float mo = hm[g], mnew = fmaxf(mo, mt);
            float ls = 0.0f;
            for (int r = lane; r < T; r += 32) {  // weights, and zeros past the tile's rows
                const float e = r < n ? expf(sp[g * T + r] - mnew) : 0.0f;
                sp[g * T + r] = e;
                ls += e;
            }
            ls = WarpSum(ls);
            if (lane == 0) {
                const float cr = mo == -INFINITY ? 0.0f : expf(mo - mnew);
                hc[g] = cr;
                hl[g] = fmaf(hl[g], cr, ls);
                hm[g] = mnew;
            }
        }
        __syncthreads();
        if (vrg < G.R) {
#pragma unroll
            for (int g = 0; g < GM; ++g)
                if (g < gcnt) {
                    const float cr = hc[g];
                    acc[g].x *= cr;
                    acc[g].y *= cr;
                    acc[g].z *= cr;
                    acc[g].w *= cr;
                }
            if (vquad) {
                // four consecutive rows: their V pieces once, then one
                // 16-byte load of the four weights per head; rows past n
                // count as zero rows (their weights are zero too)
                const int rb = 4 * vrg;
                float4 v[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int r = rb + j;
                    v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (r < n) v[j] = Lds4((r0 + r == skip_row ? vn : vt + r * hdp) + 4 * vcol);
                }
#pragma unroll
                for (int g = 0; g < GM; ++g)
                    if (g < gcnt) {
                        const float4 w = Lds4(sp + g * T + rb);
                        acc[g].x = fmaf(w.x, v[0].x, acc[g].x);
                        acc[g].y = fmaf(w.x, v[0].y, acc[g].y);
                        acc[g].z = fmaf(w.x, v[0].z, acc[g].z);
                        acc[g].w = fmaf(w.x, v[0].w, acc[g].w);
                        acc[g].x = fmaf(w.y, v[1].x, acc[g].x);
                        acc[g].y = fmaf(w.y, v[1].y, acc[g].y);
                        acc[g].z = fmaf(w.y, v[1].z, acc[g].z);
                        acc[g].w = fmaf(w.y, v[1].w, acc[g].w);
                        acc[g].x = fmaf(w.z, v[2].x, acc[g].x);
                        acc[g].y = fmaf(w.z, v[2].y, acc[g].y);
                        acc[g].z = fmaf(w.z, v[2].z, acc[g].z);
                        acc[g].w = fmaf(w.z, v[2].w, acc[g].w);
                        acc[g].x = fmaf(w.w, v[3].x, acc[g].x);
                        acc[g].y = fmaf(w.w, v[3].y, acc[g].y);
                        acc[g].z = fmaf(w.w, v[3].z, acc[g].z);
                        acc[g].w = fmaf(w.w, v[3].w, acc[g].w);
                    }
            } else {
                for (int r = vrg; r < n; r += G.R) {
                    const float4 v = Lds4((r0 + r == skip_row ? vn : vt + r * hdp) + 4 * vcol);
#pragma unroll
                    for (int g = 0; g < GM; ++g)
                        if (g < gcnt) {
                            const float w = sp[g * T + r];
                            acc[g].x = fmaf(w, v.x, acc[g].x);
                            acc[g].y = fmaf(w, v.y, acc[g].y);
                            acc[g].z = fmaf(w, v.z, acc[g].z);
                            acc[g].w = fmaf(w, v.w, acc[g].w);
                        }
                }
            }
        }
    }

    if constexpr (TMA) {
        if (t < ntiles) {
            // a tile wait gave up (status recorded): wait, bounded, for the
            // tiles still in flight into this CTA's ring, then leave
            if (tid == 0)
                for (int k = t; k < ntiles && k < t + kAttnStages - 1; ++k)
                    MbarWaitFor(&full[k % kAttnStages], (k / kAttnStages) & 1, kAttnWaitNs, nullptr);
            return;
        }
    }

    // ---- the row groups' partial outputs, summed: final output or the
    // chunk's partial (every copy has landed: each tile was waited for)
    __syncthreads();  // the ring is free (red overlays it)
    if (vrg < G.R)
#pragma unroll
        for (int g = 0; g < GM; ++g)
            if (g < gcnt) *reinterpret_cast<float4*>(red + (vrg * GM + g) * hdp + 4 * vcol) = acc[g];
    __syncthreads();
    for (int i = tid; i < gcnt * hd; i += kAttnThreads) {
        const int g = i / hd, d = i - g * hd;
        float o = 0.0f;
        for (int rg = 0; rg < G.R; ++rg) o += red[(rg * GM + g) * hdp + d];
        const int h = h0 + g;
        const float l = hl[g];
        if (p.chunks == 1) {
            p.out[(size_t(b) * p.n_heads + h) * hd + d] = l > 0.0f ? o / l : 0.0f;
        } else {
            const size_t pc = (size_t(b) * p.n_heads + h) * p.chunks + chunk;
            p.part_o[pc * hd + d] = o;
            if (d == 0) {
                p.part_ml[pc * 2] = hm[g];  // -inf for an empty chunk
                p.part_ml[pc * 2 + 1] = l;
            }
        }
    }
}

void LaunchAttention(const AttnParams& p, int batch, cudaStream_t stream, bool pdl);
// Launches AttnMergeKernel over `rows` (sequence, head) partials.
void LaunchAttnMerge(const float* part_ml, const float* part_o, int chunks, int hd, float* out, int rows,
                     cudaStream_t stream);
int AttnChunks(int max_npos, int batch, int n_kv, int hgroups, int sm_count);

}  // namespace mlb
