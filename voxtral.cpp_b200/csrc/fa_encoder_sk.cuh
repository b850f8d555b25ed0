// fa_encoder_sk.cuh — persistent tcgen05 flash attention for the
// bidirectional encoder node (src/voxtral.cpp:1611 with mask = NULL: the
// offline model's 1500-token, 20-head x 64 self-attention).
//
// The per-pair kernel (fa_prefill_sm100.cuh) gives every CTA a pair of
// 128-row Q tiles and all of their key tiles.  When that grid is more than
// one wave (two clips of the offline encoder: 240 CTAs of 12 key tiles on 148
// SMs), its last wave leaves SMs idle.  Here the grid is one CTA per SM, and the work,
// units = (batch, KV head, Q-tile pair) x key tiles flattened unit-major, is
// cut into equal contiguous ranges, one per CTA ("stream-K").  A CTA walks
// its range from the top down in segments (the key tiles of one unit it
// covers), keeping its TMEM, barriers and K/V ring across segments: the TMA
// warp loads the next segment's Q tiles as soon as the last S of the current
// one has retired and streams its K/V tiles into the same ring, and the
// tensor core starts the next segment's first S while the softmax warps
// write the previous O out.
//
// A unit split between CTAs is merged in the kernel, with no waiting in
// steady state:
//   * the CTA whose range holds the unit's LAST key tile owns it; the pieces
//     before belong to lower-numbered CTAs, for which the unit is the first
//     segment they process (ranges are walked top down);
//   * each of those writes its unnormalised (O, m, l) for both Q tiles into
//     its own workspace slot and raises one flag per Q tile (release);
//   * the owner processes the unit last, then reads the flags (acquire,
//     bounded wait) and partials of its producers and merges them in a
//     fixed order (its own piece, then the producers from the lowest key
//     tiles up): O = sum_i 2^(m_i - M) O_i, l likewise, out = O / l.
//   The owner only ever waits for lower-numbered CTAs, which were dispatched
//   before it, so the merge cannot deadlock.
//   A flag is a 64-bit word that the producer sets to a tag of its launch:
//   %gridid, the context's temporal grid-launch number (distinct for every
//   launch, graph replays included), mixed with a 64-bit constant.  An owner
//   accepts only its own launch's tag, so flags left by earlier launches and
//   whatever the caller's workspace held before never count, and no clearing
//   pass is needed between launches.
//
// Roles, TMEM layout and softmax arithmetic are those of the per-pair
// kernel's D = 64 instantiation: two softmax warpgroups (one per Q tile),
// a TMA warp, an MMA warp; S_t at columns t*128 with P aliased, O_t after the
// S block with 16 extra columns that accumulate the row sum through a
// constant block of ones; P = 2^(x*c - m) with MUFU ex2 for 5/8 of the
// column pairs and a degree-3 polynomial on the FMA pipe for the rest; lazy
// rescaling.
//
// Write-back never holds up the softmax warps: they stage a segment's O
// (normalised rows, or a producer's raw partial) in a dedicated 64 KB
// shared-memory area, in the 128-byte swizzle of the TMA boxes, and go on to
// the next segment.  A store warp issues the TMA stores (output rows through
// the destination's tensor map, partials through a map of the workspace),
// waits for them, raises a producer's flags and hands the staging area back.
#pragma once
#include "fa_prefill_sm100.cuh"

namespace vtx {

constexpr int kSkMaxCtas = 160;

struct SkArgs {
    int n_pairs;            // Q-tile pairs per (batch, KV head)
    int n_iter;             // key tiles per pair (every pair attends every key tile)
    int total;              // units x n_iter (< 2^31)
    int bound[kSkMaxCtas + 1];   // CTA c takes positions [bound[c], bound[c+1]) of the flattened work
    // producer partials, one block per (CTA, Q tile) written through tmP:
    // [D/4 + 1 column groups][128 rows][4 floats], group D/4 = (m, l, 0, 0)
    const float *part;
    unsigned long long *flags;   // one per (CTA, Q tile): the launch tag once that partial is in memory
};

template <int D> struct SkCfg {
    static_assert(D == 64, "persistent encoder kernel: head_dim 64");
    static constexpr int NQT = 2, BN = 128, STAGES = 3;
    static constexpr int TILE_BYTES = 128 * D * 2;             // one Q / K / V tile (16 KB)
    static constexpr int QBUF = NQT * TILE_BYTES;               // the two Q tiles of a pair
    static constexpr int Q_OFF = 0;
    static constexpr int K_OFF = Q_OFF + QBUF;
    static constexpr int V_OFF = K_OFF + STAGES * TILE_BYTES;
    static constexpr int ONES_OFF = V_OFF + STAGES * TILE_BYTES;
    static constexpr int BOX_BYTES = 128 * 32 * 4;              // [128 rows][32 floats] output box
    // staging, per tile: output rows as D/32 swizzled boxes, or a producer's
    // partial as [D/4 + 1][128][4] floats (one unswizzled box)
    static constexpr int PGROUPS = D / 4 + 1;
    static constexpr int STG_TILE = (D / 32) * BOX_BYTES > PGROUPS * 128 * 16 ? (D / 32) * BOX_BYTES : PGROUPS * 128 * 16;
    static constexpr int STG_OFF = ONES_OFF + 16384;
    static constexpr int BAR_OFF = STG_OFF + NQT * STG_TILE;
    // q_full, q_empty, kv_full[S], v_full[S], kv_empty[S], s_full[2], p_full[2], o_full, staged[2], stage_free[2]
    static constexpr int NBARS = 2 + 3 * STAGES + 2 * NQT + 1 + 2 * NQT;
    static constexpr int SMEM = BAR_OFF + NBARS * 8 + 16 + 1024;
    static constexpr int NTHREADS = 128 * NQT + 128;
    static constexpr int TMA_WARP = 4 * NQT, MMA_WARP = 4 * NQT + 1, STORE_WARP = 4 * NQT + 2;
    static constexpr int OC = D + 16;                           // O columns incl. the row-sum block
    static constexpr int TMEM_COLS = 512;
    __host__ __device__ static constexpr int s_col(int t) { return t * 128; }
    __host__ __device__ static constexpr int o_col(int t) { return NQT * 128 + t * OC; }
    static constexpr int REG_SOFTMAX = 224, REG_PRODUCER = 56;
    static constexpr int POLY_PAIRS = 3;
};

// error code written to PrefillArgs::err when a producer's flag never came
enum { VTX_KERR_MERGE = 6, VTX_KERR_STORE = 7 };

__device__ __forceinline__ void st_release_gpu(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// This launch's merge-flag tag (see above).
__device__ __forceinline__ unsigned long long launch_tag() {
    unsigned long long id;
    asm volatile("mov.u64 %0, %%gridid;" : "=l"(id));
    return id ^ 0x9E3779B97F4A7C15ull;
}
__device__ __forceinline__ unsigned long long ld_relaxed_gpu(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// Bounded wait (wall time, like mbar_wait) of a whole warp for a producer's
// flag: lane 0 polls with relaxed loads and, once the flag is up, issues one
// acquire fence; the warp barrier then orders every lane's later loads after
// it.  Returns the verdict in every lane.
__device__ __forceinline__ bool warp_flag_wait(const unsigned long long *f, unsigned long long tag, int *err) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) {
        if (ld_relaxed_gpu(f) != tag) {
            const uint64_t t0 = globaltimer_ns();
            for (;;) {
                __nanosleep(64);
                if (ld_relaxed_gpu(f) == tag) break;
                if (globaltimer_ns() - t0 > VTX_WAIT_NS) {
                    ok = 0;
                    break;
                }
            }
        }
        if (ok) asm volatile("fence.acq_rel.gpu;" ::: "memory");
        else if (err) atomicCAS(err, 0, VTX_KERR_MERGE);
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();
    return ok != 0;
}
__device__ __forceinline__ void tma_store_3d(const void *desc, const void *src, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(desc),
                 "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

template <int D>
__global__ void __launch_bounds__(SkCfg<D>::NTHREADS, 1)
fa_encoder_sk_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmO,
                     const __grid_constant__ CUtensorMap tmP, const PrefillArgs a, const SkArgs sk)
{
    using C = SkCfg<D>;
    constexpr int NQT = C::NQT, ST = C::STAGES, NB = D / 32;
    extern __shared__ __align__(1024) char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *q_full = bars;                       // the pair's Q tiles landed
    uint64_t *q_empty = q_full + 1;                // every S MMA reading them retired
    uint64_t *kv_full = q_empty + 1;               // [ST] K_j of a stage landed
    uint64_t *v_full = kv_full + ST;               // [ST] V_j landed
    uint64_t *kv_empty = v_full + ST;              // [ST] stage consumed
    uint64_t *s_full = kv_empty + ST;              // [NQT] S_t ready
    uint64_t *p_full = s_full + NQT;               // [NQT] P_t stored (4 warp arrivals)
    uint64_t *o_full = p_full + NQT;               // every MMA of a segment retired
    uint64_t *staged = o_full + 1;                 // [NQT] tile t's O staged (4 warp arrivals)
    uint64_t *stage_free = staged + NQT;           // [NQT] the store warp has read tile t's staging
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(stage_free + NQT);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x;
    const int c_lo = sk.bound[cta];
    const int c_hi = sk.bound[cta + 1];
    const int NI = sk.n_iter;
    const int rows_per_tile = a.tok_per_tile * a.G;

    // The segment below position `hi` of this CTA's range: unit u, key tiles
    // [ia, ie).  Returns the segment's start (the next segment's `hi`).
    auto segment = [&](int hi, int &u, int &ia, int &ie) -> int {
        u = (hi - 1) / NI;
        const int u0 = u * NI;
        const int lo = c_lo > u0 ? c_lo : u0;
        ia = lo - u0;
        ie = hi - u0;
        return lo;
    };

    if (tid == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int s = 0; s < ST; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int t = 0; t < NQT; ++t) {
            mbar_init(&s_full[t], 1);
            mbar_init(&p_full[t], 4);
            mbar_init(&staged[t], 4);
            mbar_init(&stage_free[t], 1);
        }
        mbar_init(o_full, 1);
        fence_mbar_init();
    }
    if (warp == C::MMA_WARP) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == C::TMA_WARP && lane == 0) {
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        tma_prefetch_desc(&tmQ);
    }
    if (warp == C::STORE_WARP && lane == 0) {
        tma_prefetch_desc(&tmO);
        tma_prefetch_desc(&tmP);
    }
    // constant block [128 keys][64 columns] f16 in the V tiles' swizzled
    // layout: column 0 is 1.0 (chunk 0 of key row k sits at chunk k & 7)
    for (int i = tid; i < 1024; i += C::NTHREADS) {
        const int k = i >> 3, pos = i & 7;
        *reinterpret_cast<uint4 *>(smem + C::ONES_OFF + i * 16) = make_uint4(pos == (k & 7) ? 0x3C00u : 0u, 0u, 0u, 0u);
    }
    fence_proxy_async_smem();
    grid_dep_wait();            // set-up above overlaps the previous kernel; its flags / partials are settled now
    grid_dep_launch();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4 * NQT) {
        setmaxnreg_inc<C::REG_SOFTMAX>();
        // =================== softmax warpgroups ===============================
        const int t = warp >> 2;                   // Q tile of the pair
        const int r = tid & 127;                   // row == TMEM lane
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t s_addr = tmem + lane_base + C::s_col(t);
        const uint32_t o_addr = tmem + lane_base + C::o_col(t);
        char *stg = smem + C::STG_OFF + t * C::STG_TILE;
        const float cx = a.cx;
        bool ok = true;
        int gi = 0;                                // key tiles processed by this CTA so far
        int k = 0;                                 // segments processed
        for (int hi = c_hi; hi > c_lo && ok; ++k) {
            int u, ia, ie;
            hi = segment(hi, u, ia, ie);
            const int pr = u % sk.n_pairs;
            const int gb = u / sk.n_pairs;
            const int qt = 2 * pr + t;
            const int tok = qt * a.tok_per_tile + r / a.G;
            const bool row_ok = qt < a.n_tiles_q && r < rows_per_tile && tok < a.n_q;
            const int hi_key = a.n_kv - 1;
            (void)gb;
            float m_run = -INFINITY;
            for (int it = ia; it < ie; ++it, ++gi) {
                ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], (uint32_t)(gi & 1), a.err, VTX_KERR_S));
                if (!ok) break;
                tc_fence_after();
                float s[128];
                {
                    uint32_t raw[128];
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&raw[c * 32]));
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 128; ++i) s[i] = __uint_as_float(raw[i]);
                }
                const int k0 = it * C::BN;
                // keys past the sequence (last key tile): -inf.  Padding rows
                // (past n_q: zero Q from the TMA fill) are never masked, their
                // output is dropped, so full warps never split on them.
                const bool full = !row_ok || k0 + C::BN - 1 <= hi_key;
                if (__any_sync(0xffffffffu, !full)) {
#pragma unroll
                    for (int i = 0; i < 128; ++i) s[i] = k0 + i > hi_key ? -INFINITY : s[i];
                }
                float mx8[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    mx8[q] = fmaxf(s[16 * q], s[16 * q + 1]);
#pragma unroll
                    for (int i = 2; i < 16; i += 2) mx8[q] = fmax3(mx8[q], s[16 * q + i], s[16 * q + i + 1]);
                }
                const float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                                       fmaxf(mx8[6], mx8[7])) * cx;
                bool rescale = false;
                float alpha = 1.0f;
                if (mx > m_run + 8.0f) {             // lazy rescale: only on a 2^8 jump
                    if (m_run != -INFINITY) {
                        alpha = ex2(m_run - mx);
                        rescale = it > ia;
                    }
                    m_run = mx;
                }
                const float neg_m = m_run == -INFINITY ? 0.0f : -m_run;
                const uint64_t cx2 = pk2(cx, cx), nm2 = pk2(neg_m, neg_m);
                uint32_t pk[64];
#pragma unroll
                for (int pi = 0; pi < 64; ++pi) {
                    float e0, e1;
                    upk2(ffma2(pk2(s[2 * pi], s[2 * pi + 1]), cx2, nm2), e0, e1);
                    if ((pi & 7) >= 8 - C::POLY_PAIRS) {
                        exp2_poly2(e0, e1);
                    } else {
                        e0 = ex2(e0);
                        e1 = ex2(e1);
                    }
                    pk[pi] = pack_half2(e0, e1);
                }
                tmem_st32(s_addr, *reinterpret_cast<const uint32_t(*)[32]>(&pk[0]));
                tmem_st32(s_addr + 32, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32]));
                // tcgen05.ld/st are warp-collective: the whole warp rescales if any row needs it
                if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        uint32_t o[32];
                        tmem_ld32(o_addr + c * 32, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(o_addr + c * 32, o);
                    }
                    uint32_t l1 = tmem_ld1(o_addr + D);
                    tmem_ld_wait();
                    tmem_st1(o_addr + D, __float_as_uint(__uint_as_float(l1) * alpha));
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[t]);
            }
            if (!ok) break;
            // ---- segment epilogue ---------------------------------------------
            ok = __all_sync(0xffffffffu, mbar_wait(o_full, (uint32_t)(k & 1), a.err, VTX_KERR_O));
            if (!ok) break;
            tc_fence_after();
            float o[D];
            float l_tot;
            {
                uint32_t raw[D];
#pragma unroll
                for (int c = 0; c < D / 32; ++c)
                    tmem_ld32(o_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&raw[c * 32]));
                l_tot = __uint_as_float(tmem_ld1(o_addr + D));
                tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < D; ++i) o[i] = __uint_as_float(raw[i]);
            }
            const bool producer = ie < NI;
            if (producer) {
                // this CTA holds key tiles [ia, ie) of the unit and a higher
                // CTA owns it: the raw O rows and (m, l) go out through the
                // staging area and the store warp, which raises the flag
            } else if (ia > 0) {
                // owner of a split unit: merge the producers -- the CTAs below
                // whose ranges reach into this unit -- in a fixed order (own
                // piece, then the producers from the lowest key tiles up)
                const int u0 = u * NI;
                int cf = cta;
                while (cf > 0 && sk.bound[cf] > u0) --cf;   // CTA holding key tile 0
                float m_acc = m_run;
                for (int c = cf; c < cta && ok; ++c) {
                    ok = warp_flag_wait(sk.flags + 2 * c + t, launch_tag(), a.err);
                    if (!ok) break;
                    // column group j of row r at float4 j * 128 + r: every warp
                    // load is 512 contiguous bytes
                    const float4 *po = reinterpret_cast<const float4 *>(sk.part) + (long long)(2 * c + t) * C::PGROUPS * 128 + r;
                    float4 x[D / 4];
#pragma unroll
                    for (int c4 = 0; c4 < D / 4; ++c4) x[c4] = __ldcg(po + c4 * 128);
                    const float4 ml = __ldcg(po + (D / 4) * 128);
                    const float mp = ml.x, lp = ml.y;
                    const float mn = fmaxf(m_acc, mp);
                    if (mn == -INFINITY) continue;
                    const float w_acc = m_acc == -INFINITY ? 0.0f : ex2(m_acc - mn);
                    const float w_p = mp == -INFINITY ? 0.0f : ex2(mp - mn);
                    l_tot = l_tot * w_acc + lp * w_p;
#pragma unroll
                    for (int c4 = 0; c4 < D / 4; ++c4) {
                        o[4 * c4] = o[4 * c4] * w_acc + x[c4].x * w_p;
                        o[4 * c4 + 1] = o[4 * c4 + 1] * w_acc + x[c4].y * w_p;
                        o[4 * c4 + 2] = o[4 * c4 + 2] * w_acc + x[c4].z * w_p;
                        o[4 * c4 + 3] = o[4 * c4 + 3] * w_acc + x[c4].w * w_p;
                    }
                    m_acc = mn;
                }
                if (!ok) break;
            }
            if (!producer) {
                const float inv = l_tot == 0.0f ? 0.0f : 1.0f / l_tot;
#pragma unroll
                for (int i = 0; i < D; ++i) o[i] *= inv;
            }
            if (k > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait(&stage_free[t], (uint32_t)((k - 1) & 1), a.err, VTX_KERR_STORE));
                if (!ok) break;
            }
            if (producer) {
                // partial: column group j of row r at float4 j * 128 + r
                float4 *sp = reinterpret_cast<float4 *>(stg) + r;
#pragma unroll
                for (int c4 = 0; c4 < D / 4; ++c4)
                    sp[c4 * 128] = make_float4(o[4 * c4], o[4 * c4 + 1], o[4 * c4 + 2], o[4 * c4 + 3]);
                sp[(D / 4) * 128] = make_float4(m_run, l_tot, 0.0f, 0.0f);
            } else {
                // output rows: box c holds columns [32c, 32c + 32) of the 128
                // rows, 16-byte chunk q of row r at chunk q ^ (r & 7) (conflict-free)
#pragma unroll
                for (int c = 0; c < NB; ++c)
#pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4)
                        *reinterpret_cast<float4 *>(stg + c * C::BOX_BYTES + r * 128 + ((q4 ^ (r & 7)) << 4)) =
                            make_float4(o[32 * c + 4 * q4], o[32 * c + 4 * q4 + 1], o[32 * c + 4 * q4 + 2],
                                        o[32 * c + 4 * q4 + 3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&staged[t]);
        }
    } else {
        setmaxnreg_dec<C::REG_PRODUCER>();
        if (warp == C::TMA_WARP) {
            // =================== TMA producer =================================
            if (lane == 0) {
                int gi = 0;                        // K/V tiles issued
                int k = 0;                         // Q loads issued (= segments started)
                bool good = true;
                for (int hi = c_hi; hi > c_lo && good;) {
                    int u, ia, ie;
                    hi = segment(hi, u, ia, ie);
                    const int pr = u % sk.n_pairs;
                    const int gb = u / sk.n_pairs;
                    const int g = gb % a.Hkv, b = gb / a.Hkv;
                    if (k >= 1 && !mbar_wait(q_empty, (uint32_t)((k - 1) & 1), a.err, VTX_KERR_Q)) break;
                    mbar_arrive_expect_tx(q_full, C::QBUF);
#pragma unroll
                    for (int t = 0; t < NQT; ++t)
                        tma_load_4d(smem + C::Q_OFF + t * C::TILE_BYTES, &tmQ, q_full, 0, g * a.G,
                                    (2 * pr + t) * a.tok_per_tile, b);
                    ++k;
                    const int bkv = b / a.kv_bdiv;
                    for (int it = ia; it < ie; ++it, ++gi) {
                        const int st = gi % ST;
                        if (gi >= ST && !mbar_wait(&kv_empty[st], (uint32_t)(((gi / ST) - 1) & 1), a.err, VTX_KERR_KV)) {
                            good = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&kv_full[st], C::TILE_BYTES);
                        mbar_arrive_expect_tx(&v_full[st], C::TILE_BYTES);
                        tma_load_4d(smem + C::K_OFF + st * C::TILE_BYTES, &tmK, &kv_full[st], 0, it * C::BN, g, bkv);
                        tma_load_4d(smem + C::V_OFF + st * C::TILE_BYTES, &tmV, &v_full[st], 0, it * C::BN, g, bkv);
                    }
                }
                // drain: every issued load must land before the CTA's shared
                // memory is released (already true unless a wait failed)
                for (int i = gi > ST ? gi - ST : 0; i < gi; ++i) {
                    const int st = i % ST;
                    mbar_wait(&kv_full[st], (uint32_t)((i / ST) & 1), a.err, VTX_KERR_KV);
                    mbar_wait(&v_full[st], (uint32_t)((i / ST) & 1), a.err, VTX_KERR_KV);
                }
                if (k > 0) mbar_wait(q_full, (uint32_t)((k - 1) & 1), a.err, VTX_KERR_Q);
            }
        } else if (warp == C::MMA_WARP) {
            // =================== MMA issuer ===================================
            const uint32_t lead = elect_one();
            constexpr uint32_t IDESC_QK = idesc_f16_f32(128, 128, 0, 0);
            constexpr uint32_t IDESC_PV = idesc_f16_f32(128, C::OC, 0, 1);
            constexpr uint32_t HI = (1024u >> 4) | (1u << 14) | (2u << 29);   // SBO 1024, v1, SW128
            const uint32_t sbase = smem_u32(smem);
            const uint32_t lo_q = ((sbase + C::Q_OFF) >> 4) | (1u << 16);          // LBO 16 B (K-major)
            const uint32_t lo_k = ((sbase + C::K_OFF) >> 4) | (1u << 16);
            constexpr uint32_t T16 = C::TILE_BYTES >> 4;
            auto issue_qk = [&](int t, int kst) {
                const uint32_t s_tm = tmem + C::s_col(t);
                const uint32_t q_lo = lo_q + t * T16;
                const uint32_t k_lo = lo_k + kst * T16;
                mma_f16_ss_w(lead, s_tm, desc64(q_lo, HI), desc64(k_lo, HI), IDESC_QK, 0u);
#pragma unroll
                for (int kk = 1; kk < D / 16; ++kk) {
                    const uint32_t ko = (kk * 32) >> 4;
                    mma_f16_ss_w(lead, s_tm, desc64(q_lo + ko, HI), desc64(k_lo + ko, HI), IDESC_QK, 1u);
                }
                mma_commit_w(lead, &s_full[t]);
            };
            // O_t (+)= P_t V: the leading-byte offset of the V descriptor
            // reaches the constant block of ones (row sum in column D)
            auto issue_pv = [&](int t, int vst, uint32_t acc) {
                const uint32_t p_tm = tmem + C::s_col(t);
                const uint32_t o_tm = tmem + C::o_col(t);
                const uint32_t v_lo = (((sbase + C::V_OFF) >> 4) + vst * T16) |
                                      (((uint32_t)(C::ONES_OFF - C::V_OFF) / 16u - vst * T16) << 16);
                mma_f16_ts_w(lead, o_tm, p_tm, desc64(v_lo, HI), IDESC_PV, acc);
#pragma unroll
                for (int kk = 1; kk < 8; ++kk)
                    mma_f16_ts_w(lead, o_tm, p_tm + kk * 8, desc64(v_lo + kk * (2048 >> 4), HI), IDESC_PV, 1u);
            };
            bool good = true;
            int gi0 = 0;
            int k = 0;
            for (int hi = c_hi; hi > c_lo && good; ++k) {
                int u, ia, ie;
                hi = segment(hi, u, ia, ie);
                good = __all_sync(0xffffffffu, mbar_wait(q_full, (uint32_t)(k & 1), a.err, VTX_KERR_Q));
                if (!good) break;
                tc_fence_after();
                const int n = ie - ia;
                for (int it = 0; it <= n && good; ++it) {
                    const int gi = gi0 + it;
                    const int st = gi % ST, pst = (gi + ST - 1) % ST;
                    bool v_ready = false, k_ready = false;
#pragma unroll
                    for (int t = 0; t < NQT; ++t) {
                        if (it > 0) {                    // P V of the previous key tile
                            if (!v_ready) {
                                if (!__all_sync(0xffffffffu, mbar_wait(&v_full[pst], (uint32_t)(((gi - 1) / ST) & 1),
                                                                       a.err, VTX_KERR_KV))) {
                                    good = false;
                                    break;
                                }
                                v_ready = true;
                            }
                            if (!__all_sync(0xffffffffu,
                                            mbar_wait(&p_full[t], (uint32_t)((gi - 1) & 1), a.err, VTX_KERR_P))) {
                                good = false;
                                break;
                            }
                            tc_fence_after();
                            issue_pv(t, pst, it > 1 ? 1u : 0u);
                        }
                        if (it < n) {                    // S of this key tile
                            if (!k_ready) {
                                if (!__all_sync(0xffffffffu, mbar_wait(&kv_full[st], (uint32_t)((gi / ST) & 1), a.err,
                                                                       VTX_KERR_KV))) {
                                    good = false;
                                    break;
                                }
                                tc_fence_after();
                                k_ready = true;
                            }
                            issue_qk(t, st);
                        }
                    }
                    if (!good) break;
                    if (it == n - 1) mma_commit_w(lead, q_empty);   // the Q tiles are free once these retire
                    if (it > 0) mma_commit_w(lead, &kv_empty[pst]);
                }
                mma_commit_w(lead, o_full);
                gi0 += n;
            }
            // every MMA of this CTA must be retired before TMEM is released
            if (k > 0) mbar_wait(o_full, (uint32_t)((k - 1) & 1), a.err, VTX_KERR_O);
        } else if (warp == C::STORE_WARP) {
            // =================== store warp ===================================
            // per segment and Q tile: wait for the staged rows, TMA-store them
            // (output rows, or a producer's partial), hand the staging back
            if (lane == 0) {
                bool good = true;
                int k = 0;
                for (int hi = c_hi; hi > c_lo && good; ++k) {
                    int u, ia, ie;
                    hi = segment(hi, u, ia, ie);
                    const int pr = u % sk.n_pairs;
                    const int gb = u / sk.n_pairs;
                    const int g = gb % a.Hkv, b = gb / a.Hkv;
                    const bool producer = ie < NI;
                    for (int t = 0; t < NQT && good; ++t) {
                        good = mbar_wait(&staged[t], (uint32_t)(k & 1), a.err, VTX_KERR_STORE);
                        if (!good) break;
                        const char *stg = smem + C::STG_OFF + t * C::STG_TILE;
                        const int qt = 2 * pr + t;
                        if (producer) {
                            tma_store_3d(&tmP, stg, 0, 0, (2 * cta + t) * C::PGROUPS);
                        } else if (qt < a.n_tiles_q) {
#pragma unroll
                            for (int c = 0; c < NB; ++c)
                                tma_store_4d(&tmO, stg + c * C::BOX_BYTES, c * 32, g * a.G, qt * a.tok_per_tile, b);
                        }
                        bulk_commit();
                    }
                    if (!good) break;
                    if (producer) {
                        // the partial is in memory: release it to the owner
                        bulk_wait_all_done();
                        fence_proxy_async_global();
                        __threadfence();
#pragma unroll
                        for (int t = 0; t < NQT; ++t) st_release_gpu(sk.flags + 2 * cta + t, launch_tag());
                    } else {
                        bulk_wait_read_all();
                    }
#pragma unroll
                    for (int t = 0; t < NQT; ++t) mbar_arrive(&stage_free[t]);
                }
                bulk_wait_all_done();
            }
        }
    }

    // ---- teardown -------------------------------------------------------------
    tc_fence_before();
    __syncthreads();
    if (warp == C::MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

}  // namespace vtx
