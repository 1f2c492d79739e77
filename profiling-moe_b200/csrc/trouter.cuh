// Lane-per-token router for sm_100a ("transposed" layout), included by routing.cu.
//
// A warp takes 32 tokens at a time.  Stage 1 streams the rows (coalesced, through a
// cp.async ring) and records the 16-expert group maxima of every token; stage 2 lets lane
// l rank token l on its own:
//   pass A  maxima of the 16-element groups of s = logits + bias  (max.NaN: a NaN is seen)
//   tau     the K-th largest group maximum, a lower bound of the K-th largest score
//   pass B  only groups whose maximum is >= tau are rescanned; their elements >= tau are
//           inserted into a register top-K ordered by (score desc, index asc)
// Typically K groups qualify and about K+1 elements pass, so a token costs ~90 warp
// instructions instead of the ~320 of a warp-per-token ranking; each warp needs only a
// 4-row ring and a 3 KB table of shared memory.  A row with a NaN goes to
// the exact warp-per-token path (route_exact), which gives the same answer as torch.sort.
// Included by routing.cu inside namespace kb, after route_exact, fkey, fmax_nan and
// pick_weight are defined.
#pragma once



template <int E_, int KT>
struct TCfg {
    static constexpr int GS = 16;             // elements per group
    static constexpr int G = E_ / GS;         // groups (<= 32)
    static constexpr int KM = KT ? KT : 8;    // register top-K capacity
    static_assert(E_ % 128 == 0 && G <= 32 && G >= KM, "unsupported transposed-router shape");
};

// Row-wise sink: lane holds the K picks of its own token.
template <bool SEL, bool HIST, int KM, typename WT>
__device__ __forceinline__ void put_row(int32_t* ids, WT* w, int* sel, int64_t sel_t0, int* hist,
                                        int64_t t, int K, const int (&idx)[KM],
                                        const float (&wv)[KM]) {
    int32_t* ip = ids + t * K;
    WT* wp = w + t * K;
#pragma unroll
    for (int i = 0; i < KM; ++i) {
        if (i < K) {
            ip[i] = idx[i];
            wp[i] = Elem<WT>::from_f(wv[i]);
            if constexpr (SEL) sel[(int)(t - sel_t0) * K + i] = idx[i];
            if constexpr (HIST) atomicAdd(&hist[idx[i]], 1);
        }
    }
}

// Per-warp shared memory of the hybrid router: a ring of kRing rows and the 32 x (G+1)
// group-maximum table.
constexpr int kRing = 4;
template <int E_>
__host__ __device__ constexpr size_t hwarp_smem_floats() { return (size_t)kRing * E_ + 32 * (E_ / 16 + 1); }

// Route tokens [tb0, te) of this warp in batches of 32.
//   stage 1  warp-cooperative, one token at a time: the row streams through a kRing-deep
//            cp.async ring (coalesced), s = x + b stays in registers (VEC layout, 4 experts
//            per float4), and the 16-expert group maxima (float4 max + quad shuffle) go to
//            gm[token][group].
//   stage 2  lane l ranks token l from gm[l][*]: tau, then pass B re-reads only the
//            qualifying groups of its row (L2 hits) and fills a register top-K.
// b: this lane's VEC-layout bias registers; bias_sm: the same bias in shared memory;
// wsm: this warp's hwarp_smem_floats<E_>() floats; sel_tmp: 32 ints.
template <int E_, int KT, bool SEL, bool HIST, typename WT>
__device__ void troute_range(const float* __restrict__ logits, const float (&b)[E_ / 32],
                             const float* bias_sm, int K_rt, int renorm, int64_t tb0, int64_t te,
                             float* wsm, int* sel_tmp, int32_t* ids, WT* w, int* sel,
                             int64_t sel_t0, int* hist) {
    using C = TCfg<E_, KT>;
    constexpr int VPL = E_ / 32;
    constexpr int Q = VPL / 4;          // float4 chunks per lane
    constexpr int GP = C::G + 1;        // gm row stride (odd: conflict-free column reads)
    const int K = KT ? KT : K_rt;
    const int lane = threadIdx.x & 31;
    float* ring = wsm;
    float* gm = wsm + kRing * E_;
    const float4* bias4 = reinterpret_cast<const float4*>(bias_sm);
    for (int64_t tb = tb0; tb < te; tb += 32) {
        const int nb = (int)((te - tb) < 32 ? (te - tb) : 32);
        // ---------------- stage 1 ----------------
        const float* src = logits + tb * E_ + 4 * lane;
#pragma unroll
        for (int d = 0; d < kRing; ++d) {
            if (d < nb) {
#pragma unroll
                for (int q = 0; q < Q; ++q)
                    cp_async16(ring + d * E_ + 4 * lane + 128 * q, src + (int64_t)d * E_ + 128 * q);
            }
            cp_async_commit();
        }
        for (int i = 0; i < nb; ++i) {
            cp_async_wait<kRing - 1>();
            const float* rb = ring + (i % kRing) * E_ + 4 * lane;
#pragma unroll
            for (int q = 0; q < Q; ++q) {
                const float4 x = *reinterpret_cast<const float4*>(rb + 128 * q);
                float m = fmax_nan(fmax_nan(x.x + b[4 * q + 0], x.y + b[4 * q + 1]),
                                   fmax_nan(x.z + b[4 * q + 2], x.w + b[4 * q + 3]));
                m = fmax_nan(m, __shfl_xor_sync(FULL_MASK, m, 1));
                m = fmax_nan(m, __shfl_xor_sync(FULL_MASK, m, 2));
                if ((lane & 3) == 0) gm[i * GP + (lane >> 2) + 8 * q] = m;
            }
            const int nx = i + kRing;
            if (nx < nb) {
                float* dst = ring + (i % kRing) * E_ + 4 * lane;
#pragma unroll
                for (int q = 0; q < Q; ++q)
                    cp_async16(dst + 128 * q, src + (int64_t)nx * E_ + 128 * q);
            }
            cp_async_commit();
        }
        cp_async_wait<0>();
        __syncwarp();

        // ---------------- stage 2 ----------------
        const int64_t t = tb + lane;
        const bool valid = lane < nb;
        const float* row = logits + (valid ? t : tb) * E_;
        const float4* row4 = reinterpret_cast<const float4*>(row);
        float gmax[C::G];
#pragma unroll
        for (int g = 0; g < C::G; ++g) gmax[g] = gm[lane * GP + g];
        bool nan_row = false;
        float tk[C::KM];
#pragma unroll
        for (int i = 0; i < C::KM; ++i) tk[i] = -INFINITY;
#pragma unroll
        for (int g = 0; g < C::G; ++g) {
            float v = gmax[g];
            nan_row |= (v != v);
#pragma unroll
            for (int i = 0; i < C::KM; ++i) {
                const float hi = fmaxf(tk[i], v);
                v = fminf(tk[i], v);
                tk[i] = hi;
            }
        }
        float tau = tk[0];
#pragma unroll
        for (int i = 1; i < C::KM; ++i)
            if (i == K - 1) tau = tk[i];
        const bool bad = valid && nan_row;
        if (valid && !nan_row) {
            uint32_t key[C::KM];
            int idx[C::KM];
#pragma unroll
            for (int i = 0; i < C::KM; ++i) { key[i] = 0u; idx[i] = 0; }
            unsigned gq = 0u;
#pragma unroll
            for (int g = 0; g < C::G; ++g) gq |= (gmax[g] >= tau) ? (1u << g) : 0u;
            while (gq) {
                const int g = __ffs(gq) - 1;
                gq &= gq - 1u;
                unsigned m = 0u;
                float4 xs[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) xs[q] = __ldg(row4 + g * 4 + q);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 bb = bias4[g * 4 + q];
                    m |= ((xs[q].x + bb.x) >= tau ? 1u : 0u) << (4 * q + 0);
                    m |= ((xs[q].y + bb.y) >= tau ? 1u : 0u) << (4 * q + 1);
                    m |= ((xs[q].z + bb.z) >= tau ? 1u : 0u) << (4 * q + 2);
                    m |= ((xs[q].w + bb.w) >= tau ? 1u : 0u) << (4 * q + 3);
                }
                // Candidates of this group in index order, each bubbled into the list
                // ordered by (key desc, index asc); an element displaced by a larger key
                // keeps precedence over equal keys with a higher index.
                while (m) {
                    const int k = __ffs(m) - 1;
                    m &= m - 1u;
                    int jj = g * C::GS + k;
                    uint32_t kk = fkey(__ldg(row + jj) + bias_sm[jj]);
#pragma unroll
                    for (int i = 0; i < C::KM; ++i) {
                        const bool gt = kk > key[i] || (kk == key[i] && jj < idx[i]);
                        const uint32_t ok = key[i];
                        const int oi = idx[i];
                        key[i] = gt ? kk : ok;
                        idx[i] = gt ? jj : oi;
                        kk = gt ? ok : kk;
                        jj = gt ? oi : jj;
                    }
                }
            }
            float wv[C::KM];
            float sum = 0.0f;
#pragma unroll
            for (int i = 0; i < C::KM; ++i) {
                wv[i] = 0.0f;
                if (i < K) {
                    wv[i] = 1.0f / (1.0f + expf(-__ldg(row + idx[i])));
                    sum += wv[i];
                }
            }
            if (renorm) {
                const float inv = 1.0f / (sum + 1e-20f);
#pragma unroll
                for (int i = 0; i < C::KM; ++i) wv[i] = wv[i] * inv;
            }
            put_row<SEL, HIST, C::KM, WT>(ids, w, sel, sel_t0, hist, t, K, idx, wv);
        }
        // ---------------- exact path for rows holding a NaN ----------------
        unsigned badm = __ballot_sync(FULL_MASK, bad);
        while (badm) {
            const int l = __ffs(badm) - 1;
            badm &= badm - 1u;
            const float* brow = logits + (tb + l) * E_;
            route_exact<VPL, true>(brow, bias_sm, E_, K, lane, sel_tmp);
            const int id = (lane < K) ? sel_tmp[lane] : 0;
            const float wl = pick_weight((lane < K) ? __ldg(brow + id) : 0.0f, K, lane, renorm);
            if (lane < K) {
                const int64_t tt = tb + l;
                ids[tt * K + lane] = id;
                w[tt * K + lane] = Elem<WT>::from_f(wl);
                if constexpr (SEL) sel[(int)(tt - sel_t0) * K + lane] = id;
                if constexpr (HIST) atomicAdd(&hist[id], 1);
            }
            __syncwarp();
        }
        __syncwarp();
    }
}

// Shared-memory set-up of the transposed router: the bias (canonical) once per CTA.
template <int E_>
__device__ __forceinline__ void troute_setup(const float* __restrict__ bias, float* bias_sm) {
    for (int e = threadIdx.x; e < E_; e += blockDim.x)
        bias_sm[e] = bias ? __ldg(bias + e) + 0.0f : 0.0f;
    __syncthreads();
}

// Stage 1 of a batch of nb <= 32 rows that already sit in shared memory (rows_sm, row stride
// RS floats): rows r0, r0 + rstep, ... of this warp, warp-cooperative group maxima
// (conflict-free float4 reads), two rows at a time.  gm: nb x (G+1) floats.
template <int E_, int RS>
__device__ __forceinline__ void troute_stage1_sm(const float* rows_sm, int nb, int r0, int rstep,
                                                 const float (&b)[E_ / 32], float* gm) {
    constexpr int Q = E_ / 128;
    constexpr int GP = E_ / 16 + 1;
    const int lane = threadIdx.x & 31;
    for (int i = r0; i < nb; i += 2 * rstep) {
        const int i2 = i + rstep;
        const bool two = i2 < nb;
        const float* ra = rows_sm + (size_t)i * RS + 4 * lane;
        const float* rb = rows_sm + (size_t)(two ? i2 : i) * RS + 4 * lane;
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            const float4 x = *reinterpret_cast<const float4*>(ra + 128 * q);
            const float4 y = *reinterpret_cast<const float4*>(rb + 128 * q);
            float m = fmax_nan(fmax_nan(x.x + b[4 * q + 0], x.y + b[4 * q + 1]),
                               fmax_nan(x.z + b[4 * q + 2], x.w + b[4 * q + 3]));
            float n = fmax_nan(fmax_nan(y.x + b[4 * q + 0], y.y + b[4 * q + 1]),
                               fmax_nan(y.z + b[4 * q + 2], y.w + b[4 * q + 3]));
            m = fmax_nan(m, __shfl_xor_sync(FULL_MASK, m, 1));
            n = fmax_nan(n, __shfl_xor_sync(FULL_MASK, n, 1));
            m = fmax_nan(m, __shfl_xor_sync(FULL_MASK, m, 2));
            n = fmax_nan(n, __shfl_xor_sync(FULL_MASK, n, 2));
            if ((lane & 3) == 0) {
                gm[i * GP + (lane >> 2) + 8 * q] = m;
                if (two) gm[i2 * GP + (lane >> 2) + 8 * q] = n;
            }
        }
    }
}

// Stage 2 of a batch whose rows sit in shared memory (stride RS floats; RS = E_ + 4 spreads
// the rows of a warp's lanes over the banks) and whose group maxima are in gm: lane l ranks
// token tb + l (l < nb), re-reading its qualifying groups and its weights from shared memory.
// GLOBAL: rows_sm is the batch's first row in global memory instead (stride RS = E_), read
// through the read-only path.  Rows holding a NaN take the exact path on the global row.
template <int E_, int RS, int KT, typename WT, bool GLOBAL = false>
__device__ void troute_stage2_sm(const float* rows_sm, int nb, int64_t tb,
                                 const float* __restrict__ logits, const float* bias_sm,
                                 int K_rt, int renorm, const float* gm, int* sel_tmp,
                                 int32_t* ids, WT* w, int* sel, int64_t sel_t0) {
    using C = TCfg<E_, KT>;
    constexpr int GP = C::G + 1;
    const int K = KT ? KT : K_rt;
    const int lane = threadIdx.x & 31;
    const float4* bias4 = reinterpret_cast<const float4*>(bias_sm);
    // ---------------- stage 2 ----------------
    const int64_t t = tb + lane;
    const bool valid = lane < nb;
    const float* row = rows_sm + (size_t)(valid ? lane : 0) * RS;
    const float4* row4 = reinterpret_cast<const float4*>(row);
    float gmax[C::G];
#pragma unroll
    for (int g = 0; g < C::G; ++g) gmax[g] = gm[(valid ? lane : 0) * GP + g];
    bool nan_row = false;
    float tk[C::KM];
#pragma unroll
    for (int i = 0; i < C::KM; ++i) tk[i] = -INFINITY;
#pragma unroll
    for (int g = 0; g < C::G; ++g) {
        float v = gmax[g];
        nan_row |= (v != v);
#pragma unroll
        for (int i = 0; i < C::KM; ++i) {
            const float hi = fmaxf(tk[i], v);
            v = fminf(tk[i], v);
            tk[i] = hi;
        }
    }
    float tau = tk[0];
#pragma unroll
    for (int i = 1; i < C::KM; ++i)
        if (i == K - 1) tau = tk[i];
    const bool bad = valid && nan_row;
    if (valid && !nan_row) {
        uint32_t key[C::KM];
        int idx[C::KM];
#pragma unroll
        for (int i = 0; i < C::KM; ++i) { key[i] = 0u; idx[i] = 0; }
        unsigned gq = 0u;
#pragma unroll
        for (int g = 0; g < C::G; ++g) gq |= (gmax[g] >= tau) ? (1u << g) : 0u;
        while (gq) {
            const int g = __ffs(gq) - 1;
            gq &= gq - 1u;
            unsigned m = 0u;
            float xs[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 x4 = GLOBAL ? __ldg(row4 + g * 4 + q) : row4[g * 4 + q];
                const float4 bb = bias4[g * 4 + q];
                xs[4 * q + 0] = x4.x + bb.x;
                xs[4 * q + 1] = x4.y + bb.y;
                xs[4 * q + 2] = x4.z + bb.z;
                xs[4 * q + 3] = x4.w + bb.w;
            }
#pragma unroll
            for (int k = 0; k < 16; ++k) m |= (xs[k] >= tau ? 1u : 0u) << k;
            // Candidates of this group in index order, each bubbled into the list ordered by
            // (key desc, index asc); a displaced element keeps precedence over equal keys
            // with a higher index.
            while (m) {
                const int k = __ffs(m) - 1;
                m &= m - 1u;
                int jj = g * C::GS + k;
                uint32_t kk = fkey((GLOBAL ? __ldg(row + jj) : row[jj]) + bias_sm[jj]);
#pragma unroll
                for (int i = 0; i < C::KM; ++i) {
                    const bool gt = kk > key[i] || (kk == key[i] && jj < idx[i]);
                    const uint32_t ok = key[i];
                    const int oi = idx[i];
                    key[i] = gt ? kk : ok;
                    idx[i] = gt ? jj : oi;
                    kk = gt ? ok : kk;
                    jj = gt ? oi : jj;
                }
            }
        }
        float wv[C::KM];
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < C::KM; ++i) {
            wv[i] = 0.0f;
            if (i < K) {
                wv[i] = sigmoid_acc(GLOBAL ? __ldg(row + idx[i]) : row[idx[i]]);
                sum += wv[i];
            }
        }
        if (renorm) {
            const float inv = 1.0f / (sum + 1e-20f);
#pragma unroll
            for (int i = 0; i < C::KM; ++i) wv[i] = wv[i] * inv;
        }
        put_row<true, false, C::KM, WT>(ids, w, sel, sel_t0, nullptr, t, K, idx, wv);
    }
    // ---------------- exact path for rows holding a NaN ----------------
    unsigned badm = __ballot_sync(FULL_MASK, bad);
    while (badm) {
        const int l = __ffs(badm) - 1;
        badm &= badm - 1u;
        const float* brow = logits + (tb + l) * E_;
        route_exact<E_ / 32, true>(brow, bias_sm, E_, K, lane, sel_tmp);
        const int id = (lane < K) ? sel_tmp[lane] : 0;
        const float wl = pick_weight((lane < K) ? __ldg(brow + id) : 0.0f, K, lane, renorm);
        if (lane < K) {
            const int64_t tt = tb + l;
            ids[tt * K + lane] = id;
            w[tt * K + lane] = Elem<WT>::from_f(wl);
            sel[(int)(tt - sel_t0) * K + lane] = id;
        }
        __syncwarp();
    }
    __syncwarp();
}
