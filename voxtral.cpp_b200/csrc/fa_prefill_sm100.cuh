// fa_prefill_sm100.cuh — tensor-core flash attention for sm_100a (tcgen05).
//
// The encoder node (src/voxtral.cpp:1611: 1500 tokens per chunk, head_dim 64,
// bidirectional or causal + 750 window) and the decoder prefill node
// (src/voxtral.cpp:1802: GQA 32/8, head_dim 128, causal) are compute-bound.
// One CTA owns NQT 128-row Q tiles of one KV head (GQA: the G query heads of
// the group are packed into the rows, row = token * G + head-in-group, so
// every K/V tile feeds all of them) and walks the key tiles.  Warp roles, one
// warpgroup per Q tile plus one producer warpgroup:
//
//   WG t < NQT      softmax of Q tile t, one thread per row (= TMEM lane):
//                   tcgen05.ld S, max, P = 2^(x*c - m) (MUFU ex2 for most
//                   columns, a degree-3 polynomial on the FMA pipe for the
//                   rest), lazy rescaling (only when the row max grows by more
//                   than 2^8), P packed to half into its TMEM columns.
//   WG NQT warp 0   TMA producer: the f16 Q tiles first (when Q is
//                   TMA-describable), then K_j, V_j (128 keys x D, 128-byte
//                   swizzle) into a STAGES-deep shared-memory ring (one
//                   mbarrier tx count for K, one for V, per stage)
//   WG NQT warp 1   MMA issuer (one thread): S_t = Q_t K_j^T  (SS, f16->f32,
//                   TMEM), then O_t += P_t V_j with P read from TMEM (TS)
//
// With NQT = 2 the two softmax warpgroups share the SM: while one computes its
// softmax the tensor core runs the other tile's PV and next S.  The producer
// warpgroup gives registers to the softmax warpgroups (setmaxnreg).
//
// TMEM columns, look-ahead layout (D = 128 with NQT = 1): per tile S_t (128),
// P_t (64, f16 pairs), O_t (D).  The softmax releases S_t as soon as it sits
// in registers, so S_t(j+1) = Q_t K_{j+1}^T runs during the softmax of tile
// j and the softmax warps never wait for the tensor core in steady state.
// Otherwise P_t aliases the first 64 columns of S_t and O_t sits after the S
// block: D = 128 with NQT = 2 (640 columns would be needed), and D = 64, where
// O_t carries 16 extra columns for the tensor-core row sum (2 x 272 > 512);
// measured, the row sum on the tensor core is worth more than the look-ahead
// for D = 64, whose softmax instruction stream is the bound either way.  Causal / windowed
// key tiles outside every row's range are never loaded.  Numerics: Q and P
// in f16 (Q is rounded to half exactly as ggml rounds Q for an F16 K), fp32
// accumulation of S and O.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "vtx_ptx.cuh"

namespace vtx {

struct PrefillArgs {
    const char *q; int q_f16; long long q_nb1, q_nb2, q_nb3;
    const char *mask; long long m_nb1, m_nb2, m_nb3; int m_ne2, m_ne3;
    char *dst; long long d_nb1, d_nb2, d_nb3;
    int n_q, n_kv, Hq, Hkv, G, B;
    int tok_per_tile, n_tiles_q, n_cta_q;
    int kv_bdiv;
    // Pre-exponent value x and multiplier cx, P = 2^(x*cx - m):
    //   fused (softcap == 0, scale > 0): x = s + (slope/scale)*mask, cx = scale*log2(e)
    //   otherwise: x = logit (softcap*tanh(s*qk_scale) or s*scale) + slope*mask, cx = log2(e)
    int fused;
    float cx;
    float qk_scale, softcap, scale;
    float max_bias, m0, m1; int n_head_log2;
    int causal, window;
    int q_quant8;             // K was Q8_0: quantize Q rows like ggml's from_float
    int o_tma;                // dst written by TMA stores through tmO (aligned F32 dst)
    int *err;
    int lpt;                  // causal launches: longest Q-tile groups first (see the kernel)
    int q_tma;                // f16 Q tiles loaded by TMA through tmQ (else copied by the softmax warps)
    int o_f16;                // dst is F16 (with o_tma): boxes of 64 halves, rounded to nearest even
};

template <int D, int NQT> struct PrefillCfg {
    static constexpr int BM = 128, BN = 128;
    static constexpr int STAGES = D == 64 ? 3 : 2;
    static constexpr int SUB = D / 64;                         // 64-column swizzle sub-tiles
    static constexpr int TILE_BYTES = 128 * D * 2;             // one Q / K / V tile
    static constexpr int Q_OFF = 0;
    static constexpr int K_OFF = Q_OFF + NQT * TILE_BYTES;
    static constexpr int V_OFF = K_OFF + STAGES * TILE_BYTES;
    // Row sums by the tensor core (D = 64): the P V product runs with N = D + 16,
    // the extra 16 columns of "V" being a constant block whose first column is
    // 1, so O column D accumulates sum_j P_ij and the softmax warps spend no
    // adds on it.  The block follows the V ring and is reached through the
    // descriptor's leading-byte offset (the distance between 64-column blocks).
    static constexpr bool ROWSUM = D == 64;
    static constexpr int OC = D + (ROWSUM ? 16 : 0);          // O accumulator columns
    static constexpr int ONES_OFF = V_OFF + STAGES * TILE_BYTES;
    static constexpr int BAR_OFF = ONES_OFF + (ROWSUM ? 16384 : 0);
    // Look-ahead (LA): when every tile can own S (128 columns), P (64) and O
    // (D) in TMEM, P gets its own columns and Q K^T of the next key tile runs
    // while the softmax of the current one is still computing.  Otherwise P
    // aliases S and the next S waits for P V.
    static constexpr bool LA = !ROWSUM && NQT * (128 + 64 + D) <= 512;
    static constexpr int NBARS = 1 + 3 * STAGES + 4 * NQT + 1 + NQT;
    static constexpr int SMEM = BAR_OFF + NBARS * 8 + 16 + 1024;   // +1024 alignment slack
    static constexpr int NTHREADS = 128 * NQT + 128;
    static constexpr int TMA_WARP = 4 * NQT, MMA_WARP = 4 * NQT + 1;
    static constexpr int TMEM_USED = LA ? NQT * (192 + D) : NQT * (128 + OC);
    static constexpr int TMEM_COLS = TMEM_USED <= 256 ? 256 : 512;
    __host__ __device__ static constexpr int s_col(int t) { return LA ? t * (192 + D) : t * 128; }
    __host__ __device__ static constexpr int p_col(int t) { return LA ? s_col(t) + 128 : s_col(t); }
    __host__ __device__ static constexpr int o_col(int t) { return LA ? s_col(t) + 192 : NQT * 128 + t * OC; }
    // register split (NQT = 2: 384 threads launched at 168 registers)
    static constexpr int REG_SOFTMAX = 224, REG_PRODUCER = 56;
    // out of every 8 column pairs, POLY_PAIRS use the FMA-pipe exp2
#ifdef VTX_POLY_PAIRS
    static constexpr int POLY_PAIRS = VTX_POLY_PAIRS;
#else
    static constexpr int POLY_PAIRS = D == 64 ? 3 : 2;
#endif
};

// error codes written to PrefillArgs::err
enum { VTX_KERR_Q = 1, VTX_KERR_KV = 2, VTX_KERR_S = 3, VTX_KERR_P = 4, VTX_KERR_O = 5 };

// ---- packed f32x2 arithmetic (sm_100) ---------------------------------------
__device__ __forceinline__ uint64_t pk2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk2(uint64_t r, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fsub2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// 2^x on the FMA pipe for a pair (x <= ~8 here).  Cody-Waite style range
// reduction x = j + f, j = round(x), |f| <= 1/2, via the 1.5*2^23 rounding
// constant; 2^f by a degree-3 polynomial fitted here for minimum relative
// error on [-1/2, 1/2] (max rel. error 7.5e-5, below half an f16 ulp, the
// precision P is stored in); 2^j added to the exponent field.  x is clamped at
// -125 so the exponent never leaves the normal range (2^-125 rounds to 0 in
// the f16 P anyway).
__device__ __forceinline__ void exp2_poly2(float &a, float &b) {
    const float kRound = 12582912.0f;                    // 1.5 * 2^23
    a = fmaxf(a, -125.0f);
    b = fmaxf(b, -125.0f);
    const uint64_t x = pk2(a, b);
    const uint64_t t = fadd2(x, pk2(kRound, kRound));
    const uint64_t j = fadd2(t, pk2(-kRound, -kRound));
    const uint64_t f = fsub2(x, j);
    uint64_t p = ffma2(pk2(0.055171773f, 0.055171773f), f, pk2(0.24261115f, 0.24261115f));
    p = ffma2(p, f, pk2(0.69326097f, 0.69326097f));
    p = ffma2(p, f, pk2(0.99992806f, 0.99992806f));
    float pa, pb, ta, tb;
    upk2(p, pa, pb);
    upk2(t, ta, tb);
    a = __int_as_float(__float_as_int(pa) + (__float_as_int(ta) << 23));
    b = __int_as_float(__float_as_int(pb) + (__float_as_int(tb) << 23));
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
__device__ __forceinline__ uint64_t desc64(uint32_t lo, uint32_t hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}

template <int N>
__device__ __forceinline__ void setmaxnreg_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }

// HAS_MASK: an explicit F16 mask tensor is applied.  UNFUSED: softcap or a
// non-positive scale (logits formed before the exponent); a template flag so
// the common instantiation carries none of that code (the softmax loop is
// fully unrolled, and its size is what the instruction cache sees).
// OF16: the result is written as F16 (rounded to nearest even) through an F16
// output map, boxes of 64 halves; a template flag so the F32 instantiations
// carry none of that code.
template <int D, int NQT, bool HAS_MASK, bool UNFUSED, bool CSL = false, bool OF16 = false>
__global__ void __launch_bounds__(PrefillCfg<D, NQT>::NTHREADS, 1)
fa_prefill_sm100_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                        const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmQ,
                        const PrefillArgs a)
{
    using C = PrefillCfg<D, NQT>;
    extern __shared__ __align__(1024) char smem_raw[];
    char *smem = reinterpret_cast<char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *q_full = bars;
    uint64_t *kv_full = bars + 1;                  // K_j of a stage landed (V_j: v_full)
    uint64_t *kv_empty = kv_full + C::STAGES;
    uint64_t *s_full = kv_empty + C::STAGES;
    uint64_t *p_full = s_full + NQT;
    uint64_t *s_free = p_full + NQT;               // LA: S_t copied to registers, may be overwritten
    uint64_t *pv_done = s_free + NQT;              // LA: O_t += P_t V done, P_t may be rewritten
    uint64_t *o_full = pv_done + NQT;
    uint64_t *v_full = o_full + 1;                 // V_j of a stage landed
    uint64_t *o_tile = v_full + C::STAGES;         // EARLY_O: every S and tile t's last P V retired
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(o_tile + NQT);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // CSL: the instantiation for causal launches with the causal/window flags
    // (no mask tensor, no softcap) that are windowed or more than one wave
    // (measured: a single-wave plain causal launch gains nothing from it).
    // Its CTAs' key ranges grow with their Q tiles, and it differs in two ways:
    //   * a.lpt (more than one wave): grid (groups x Hkv, 1, B) taken
    //     group-major from the last group of Q tiles, so every head's longest
    //     CTAs are dispatched first and the short ones fill the tail
    //     (longest-first list scheduling); otherwise, as for every other
    //     launch, grid (groups, Hkv, B) with a head's CTAs adjacent;
    //   * each Q tile runs only over its own key tiles (tile_iters below),
    //     not over the union of the CTA's tiles.
    // EARLY_O (P aliasing S): tile t's write-back starts when its own last
    // P V has retired (o_tile[t]), while the other tile's last softmax and
    // P V still run.  When every Q tile walks the same key tiles, the MMA
    // issuer puts every S of the CTA before the first tile's last P V, so by
    // then the Q tiles and the K ring -- tile 0's and tile 1's staging -- are
    // idle; the pending P V reads only the V ring and the constant block.
    // CSL (a tile's own key range, the later tile's reaching further): the
    // later tile may still run S over Q_1 and the K ring, so tile 0 stages in
    // its own Q tile, one TILE_BYTES group of boxes at a time (TMA
    // write-back only; the row-store write-back waits for every MMA).
    constexpr bool EARLY_O = !C::LA;
    const int b = blockIdx.z;
    const bool lpt = CSL && a.lpt;
    const int g = lpt ? (int)(blockIdx.x % a.Hkv) : (int)blockIdx.y;
    const int qt0 = (lpt ? a.n_cta_q - 1 - (int)(blockIdx.x / a.Hkv) : (int)blockIdx.x) * NQT;
    const int rows_per_tile = a.tok_per_tile * a.G;
    const int off = a.n_kv - a.n_q;

    // ---- key-tile range shared by all roles --------------------------------
    const int tok_first = qt0 * a.tok_per_tile;
    const int tok_last = min(a.n_q - 1, (min(qt0 + NQT, a.n_tiles_q)) * a.tok_per_tile - 1);
    int kv_lo = 0, kv_hi = a.n_kv - 1;
    if (a.causal) {
        kv_hi = min(kv_hi, tok_last + off);
        if (a.window > 0) kv_lo = max(0, tok_first + off - (a.window - 1));
    }
    const int j_begin = kv_lo / C::BN;
    const int j_end = kv_hi >= kv_lo ? kv_hi / C::BN + 1 : j_begin;
    const int n_iter = j_end - j_begin;
    // Q tile t iterates over it in [lo_it, hi_it) of the CTA's key tiles.
    // CSL: a tile's own range -- in a window or causal pair the first tile
    // needs none of the union's last key tile (wholly in its future) and the
    // second none of its first (wholly before its window).  A tile past the
    // sequence has none.  Other launches: the whole range.
    auto tile_iters = [&](int t, int &lo_it, int &hi_it) {
        lo_it = 0;
        hi_it = n_iter;
        if constexpr (CSL) {
            const int qt = qt0 + t;
            const int tf = qt * a.tok_per_tile;
            const int tl = min(a.n_q - 1, (qt + 1) * a.tok_per_tile - 1);
            const int lo = a.window > 0 ? max(0, tf + off - (a.window - 1)) : 0;
            const int hi = min(a.n_kv - 1, tl + off);
            if (qt >= a.n_tiles_q || tf > tl || hi < lo) {
                hi_it = 0;
            } else {
                lo_it = max(0, lo / C::BN - j_begin);
                hi_it = min(n_iter, hi / C::BN + 1 - j_begin);
            }
        }
    };

    if (tid == 0) {
        mbar_init(q_full, a.q_tma ? 1 : 4 * NQT);   // the TMA thread, or one arrival per softmax warp
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int t = 0; t < NQT; ++t) {
            mbar_init(&s_full[t], 1);
            mbar_init(&p_full[t], 4);
            mbar_init(&s_free[t], 4);
            mbar_init(&pv_done[t], 1);
        }
        mbar_init(o_full, 1);
        for (int t = 0; t < NQT; ++t) mbar_init(&o_tile[t], 1);
        fence_mbar_init();
    }
    if (warp == C::MMA_WARP) {             // MMA warp owns the TMEM allocation
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == C::TMA_WARP && lane == 0) {
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        if (a.q_tma) tma_prefetch_desc(&tmQ);
    }
    grid_dep_wait();            // barriers, TMEM and the constant block above overlap the previous kernel
    grid_dep_launch();
    if constexpr (C::ROWSUM) {
        // constant block [128 keys][64 columns] f16 in the V tiles' 128-byte
        // swizzled layout: column 0 is 1.0 (16-byte chunk 0 of key row k sits at
        // chunk k & 7), everything else 0
        for (int i = tid; i < 1024; i += C::NTHREADS) {
            const int k = i >> 3, pos = i & 7;
            *reinterpret_cast<uint4 *>(smem + C::ONES_OFF + i * 16) =
                make_uint4(pos == (k & 7) ? 0x3C00u : 0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4 * NQT) {
        if (NQT == 2) setmaxnreg_inc<C::REG_SOFTMAX>();
        // =================== softmax warpgroups ===============================
        bool ok = true;
        const int t = warp >> 2;                   // Q tile within the CTA
        const int r = tid & 127;                   // row == TMEM lane
        const int qt = qt0 + t;
        const int tok = qt * a.tok_per_tile + r / a.G;
        const int head = g * a.G + r % a.G;
        const bool row_ok = qt < a.n_tiles_q && r < rows_per_tile && tok < a.n_q;
        int lo = 1, hi = 0;
        if (row_ok) {
            lo = 0;
            hi = a.n_kv - 1;
            if (a.causal) {
                hi = min(hi, tok + off);
                if (a.window > 0) lo = max(0, tok + off - (a.window - 1));
            }
        }
        // Q tile -> f16 -> swizzled smem (K-major, 128B swizzle, 64-col sub-tiles).
        // f16 Q that a tensor map describes arrives by TMA (a.q_tma, issued by
        // the producer ahead of the K/V stages).  Other f16 Q is copied by the
        // warpgroup in 16-byte chunks, consecutive
        // threads taking consecutive chunks of a row, so a warp's load touches
        // 4 rows (D = 64) instead of 32.  F32 Q (converted) and Q quantised for
        // a Q8_0 K are read a row per thread.  Every load is issued before any
        // store (the stores go through a generic pointer, so a load after them
        // could not be hoisted and would pay its own DRAM latency).
        if (a.q_tma) {
            // the TMA producer loads this tile (rows past the sequence read as zeros)
        } else if (!a.q_quant8 && a.q_f16) {
            constexpr int CPR = D / 8;                          // 16-byte f16 chunks per row
            constexpr int PER = 128 * CPR / 128;                // chunks per thread
            char *qtile = smem + C::Q_OFF + t * C::TILE_BYTES;
            // addresses first; a chunk past the sequence reads the tensor's first
            // row (always valid) and is zeroed afterwards, so the loads carry no
            // branches and all of a thread's loads are in flight together
            // thread r takes chunk r % CPR of rows r / CPR + i * RS; when the group
            // size divides RS the later rows are the same head RS / G tokens on
            // (one division per thread instead of one per chunk)
            constexpr int RS = 128 / CPR;                       // rows per step
            const int row0 = r / CPR, c = r % CPR;
            const bool step_div = RS % a.G == 0;
            const int tok0 = qt * a.tok_per_tile + row0 / a.G, head0 = g * a.G + row0 % a.G;
            const int tstep = step_div ? RS / a.G : 0;
            const char *src[PER];
            bool valid[PER];
#pragma unroll
            for (int i = 0; i < PER; ++i) {
                const int row = row0 + i * RS;
                const int ctok = step_div ? tok0 + i * tstep : qt * a.tok_per_tile + row / a.G;
                const int chead = step_div ? head0 : g * a.G + row % a.G;
                valid[i] = qt < a.n_tiles_q && row < rows_per_tile && ctok < a.n_q;
                src[i] = valid[i] ? a.q + (long long)ctok * a.q_nb1 + (long long)chead * a.q_nb2 +
                                        (long long)b * a.q_nb3 + c * 16
                                  : a.q;
            }
            uint4 pkc[PER];
#pragma unroll
            for (int i = 0; i < PER; ++i) pkc[i] = *reinterpret_cast<const uint4 *>(src[i]);
#pragma unroll
            for (int i = 0; i < PER; ++i)
                if (!valid[i]) pkc[i] = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int i = 0; i < PER; ++i) {
                const int row = row0 + i * RS, sub = c >> 3, cc = c & 7;
                *reinterpret_cast<uint4 *>(qtile + sub * 16384 + row * 128 + ((cc ^ (row & 7)) << 4)) = pkc[i];
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(q_full);
        } else {
            char *qtile = smem + C::Q_OFF + t * C::TILE_BYTES;
            const char *src = a.q + (long long)tok * a.q_nb1 + (long long)head * a.q_nb2 + (long long)b * a.q_nb3;
            float f[D];
            if (row_ok) {
                if (a.q_f16) {
                    uint4 raw[D / 8];
#pragma unroll
                    for (int c = 0; c < D / 8; ++c) raw[c] = *reinterpret_cast<const uint4 *>(src + c * 16);
#pragma unroll
                    for (int c = 0; c < D / 8; ++c) {
                        const __half2 *h = reinterpret_cast<const __half2 *>(&raw[c]);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float2 x = __half22float2(h[i]);
                            f[8 * c + 2 * i] = x.x;
                            f[8 * c + 2 * i + 1] = x.y;
                        }
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < D / 4; ++c) {
                        const float4 x = *reinterpret_cast<const float4 *>(src + c * 16);
                        f[4 * c] = x.x; f[4 * c + 1] = x.y; f[4 * c + 2] = x.z; f[4 * c + 3] = x.w;
                    }
                }
                if (a.q_quant8) {
                    // K is Q8_0 in the caller's tensor: ggml quantizes Q to Q8_0
                    // (per 32 values: d = amax/127, q = rne(x*127/amax)) before
                    // the dot; reproduce that and feed d*q (as half) to the MMA.
#pragma unroll
                    for (int blk = 0; blk < D / 32; ++blk) {
                        float amax = 0.0f;
#pragma unroll
                        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(f[32 * blk + i]));
                        const float dq = __half2float(__float2half_rn(amax / 127.0f));
                        const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
#pragma unroll
                        for (int i = 0; i < 32; ++i) f[32 * blk + i] = dq * (float)__float2int_rn(f[32 * blk + i] * id);
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < D; ++i) f[i] = 0.0f;
            }
#pragma unroll
            for (int c = 0; c < D / 8; ++c) {
                uint4 pk;
                pk.x = pack_half2(f[8 * c], f[8 * c + 1]); pk.y = pack_half2(f[8 * c + 2], f[8 * c + 3]);
                pk.z = pack_half2(f[8 * c + 4], f[8 * c + 5]); pk.w = pack_half2(f[8 * c + 6], f[8 * c + 7]);
                const int sub = c >> 3, cc = c & 7;
                *reinterpret_cast<uint4 *>(qtile + sub * 16384 + r * 128 + ((cc ^ (r & 7)) << 4)) = pk;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(q_full);
        }
        float slope = 1.0f;
        if (a.max_bias > 0.0f)
            slope = head < a.n_head_log2 ? powf(a.m0, (float)(head + 1))
                                         : powf(a.m1, (float)(2 * (head - a.n_head_log2) + 1));
        const float mask_mul = UNFUSED ? slope : slope / a.scale;
        const char *mrow = nullptr;
        if (HAS_MASK && row_ok)
            mrow = a.mask + (long long)tok * a.m_nb1 + (long long)(head % a.m_ne2) * a.m_nb2 +
                   (long long)(b % a.m_ne3) * a.m_nb3;

        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t s_addr = tmem + lane_base + C::s_col(t);
        const uint32_t p_addr = tmem + lane_base + C::p_col(t);
        const uint32_t o_addr = tmem + lane_base + C::o_col(t);
        const float cx = a.cx;
        float m_run = -INFINITY, l_run = 0.0f;

        int t_lo, t_hi;
        tile_iters(t, t_lo, t_hi);
        const int t_iters = t_hi - t_lo;
        for (int it = t_lo; it < t_hi && ok; ++it) {
            const int j = j_begin + it;
            ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], (it - t_lo) & 1, a.err, VTX_KERR_S));
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
            if constexpr (C::LA) {                   // S_t is in registers: the next Q K^T may overwrite it
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[t]);
            }
            const int k0 = j * C::BN;
            if (UNFUSED) {
#pragma unroll
                for (int i = 0; i < 128; ++i)
                    s[i] = a.softcap != 0.0f ? a.softcap * tanhf(s[i] * a.qk_scale) : s[i] * a.scale;
            }
            // Padding rows (row_ok false) never need masking: their output is
            // dropped.  The masking pass runs warp-uniformly so rows that are
            // fully inside their key range never split the warp.
            const bool full = !HAS_MASK && (!row_ok || (k0 >= lo && k0 + C::BN - 1 <= hi));
            if (__any_sync(0xffffffffu, !full)) {
#pragma unroll
                for (int i = 0; i < 128; ++i) {
                    const int key = k0 + i;
                    float x = s[i];
                    if (HAS_MASK && key >= lo && key <= hi)
                        x = fmaf(mask_mul, __half2float(reinterpret_cast<const __half *>(mrow)[key]), x);
                    s[i] = (key < lo || key > hi) ? -INFINITY : x;
                }
            }
            // row max (tree over 8 independent chains)
            // row max: 8 independent chains of 3-input max
            float mx8[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                mx8[k] = fmaxf(s[16 * k], s[16 * k + 1]);
#pragma unroll
                for (int i = 2; i < 16; i += 2) mx8[k] = fmax3(mx8[k], s[16 * k + i], s[16 * k + i + 1]);
            }
            const float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]),
                                   fmaxf(mx8[6], mx8[7])) * cx;
            bool rescale = false;
            float alpha = 1.0f;
            if (mx > m_run + 8.0f) {                 // lazy rescale: only on a 2^8 jump
                if (m_run != -INFINITY) {
                    alpha = ex2(m_run - mx);
                    rescale = it > t_lo;
                }
                m_run = mx;
                l_run *= alpha;
            }
            const float neg_m = m_run == -INFINITY ? 0.0f : -m_run;
            // P = 2^(x*cx - m): MUFU for most pairs, FMA-pipe polynomial for the rest
            // With the tensor-core row sum each pair is packed to halves as soon
            // as it is computed; otherwise the f32 values are summed first.
            uint64_t sum2[4] = {0ull, 0ull, 0ull, 0ull};
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
                if (C::ROWSUM) {
                    pk[pi] = pack_half2(e0, e1);
                } else {
                    s[2 * pi] = e0;
                    s[2 * pi + 1] = e1;
                    sum2[pi & 3] = fadd2(sum2[pi & 3], pk2(e0, e1));
                }
            }
            if (!C::ROWSUM) {
                const uint64_t s01 = fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3]));
                float sa, sb;
                upk2(s01, sa, sb);
                l_run += sa + sb;
            }
            // P packed to half pairs before any wait, so the conversions can be
            // scheduled among the exponentials
            if (!C::ROWSUM) {
#pragma unroll
                for (int i = 0; i < 64; ++i) pk[i] = pack_half2(s[2 * i], s[2 * i + 1]);
            }
            if (C::LA && it > t_lo) {               // P_t and O_t are free once the previous P V retired
                ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[t], (it - t_lo - 1) & 1, a.err, VTX_KERR_O));
                if (!ok) break;
                tc_fence_after();
            }
            tmem_st32(p_addr, *reinterpret_cast<const uint32_t(*)[32]>(&pk[0]));
            tmem_st32(p_addr + 32, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32]));
            // tcgen05.ld/st are warp-collective (.sync.aligned): the whole warp
            // rescales if any of its rows needs it (alpha == 1 for the others).
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
                if constexpr (C::ROWSUM) {            // the row-sum column (columns D+1.. stay 0)
                    uint32_t l1 = tmem_ld1(o_addr + D);
                    tmem_ld_wait();
                    tmem_st1(o_addr + D, __float_as_uint(__uint_as_float(l1) * alpha));
                }
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t]);   // per-warp arrival
        }
        // ---- epilogue: O / l -> dst ------------------------------------------
        const bool early_o = EARLY_O && (!CSL || a.o_tma);
        if (ok && n_iter > 0)
            ok = __all_sync(0xffffffffu, mbar_wait(early_o ? &o_tile[t] : o_full, 0, a.err, VTX_KERR_O));
        // After o_full every MMA has retired and every TMA load has landed, so
        // the Q tiles and the K/V ring are free to stage O; after o_tile[t]
        // (EARLY_O) every S has, so the Q tiles and the K ring are.
        if (a.o_tma) {
            // Staged as D/32 boxes of [128 rows][32 floats] per tile in the 128-byte
            // swizzled layout of the output tensor map (conflict-free: a row's
            // 16-byte chunk c sits at chunk c ^ (row & 7)), then written by one
            // TMA store per box; rows past the end of the sequence are clipped by
            // the hardware.
            static_assert(NQT * (D / 32) * 16384 <= C::BAR_OFF, "O staging overlaps the barriers");
            const bool own_q = CSL && EARLY_O && NQT == 2 && t == 0;
            char *st = own_q ? smem + C::Q_OFF : smem + C::Q_OFF + t * (D / 32) * 16384;
            float inv = 0.0f;
            if (ok) {
                tc_fence_after();
                if constexpr (C::ROWSUM) {
                    if (t_iters > 0) {
                        l_run = __uint_as_float(tmem_ld1(o_addr + D));
                        tmem_ld_wait();
                    }
                }
                inv = l_run == 0.0f ? 0.0f : 1.0f / l_run;
            }
            const bool store = __all_sync(0xffffffffu, ok) && r == 0 && qt < a.n_tiles_q;
            if constexpr (OF16) {
                // F16 result: boxes of [128 rows][64 halves], same swizzle
#pragma unroll
                for (int c = 0; c < D / 64; ++c) {
                    if (ok) {
                        // 32 columns (four 16-byte chunks of halves) at a time
                        for (int hh = 0; hh < 2; ++hh) {
                            uint32_t o[32];
                            if (t_iters > 0) {
                                tmem_ld32(o_addr + c * 64 + hh * 32, o);
                                tmem_ld_wait();
                            } else {
#pragma unroll
                                for (int i = 0; i < 32; ++i) o[i] = 0u;
                            }
#pragma unroll
                            for (int q4 = 0; q4 < 4; ++q4) {
                                const int q8 = hh * 4 + q4;
                                *reinterpret_cast<uint4 *>(st + c * 16384 + r * 128 + ((q8 ^ (r & 7)) << 4)) = make_uint4(
                                    pack_half2(__uint_as_float(o[8 * q4]) * inv, __uint_as_float(o[8 * q4 + 1]) * inv),
                                    pack_half2(__uint_as_float(o[8 * q4 + 2]) * inv, __uint_as_float(o[8 * q4 + 3]) * inv),
                                    pack_half2(__uint_as_float(o[8 * q4 + 4]) * inv, __uint_as_float(o[8 * q4 + 5]) * inv),
                                    pack_half2(__uint_as_float(o[8 * q4 + 6]) * inv, __uint_as_float(o[8 * q4 + 7]) * inv));
                            }
                        }
                    }
                    fence_proxy_async_smem();
                    asm volatile("bar.sync %0, 128;" ::"r"(1 + t) : "memory");   // box c of this tile is staged
                    if (store) {
                        tma_store_4d(&tmO, st + c * 16384, c * 64, g * a.G, qt * a.tok_per_tile, b);
                        bulk_commit();
                    }
                }
            }
            // one box at a time: its store is issued as soon as it is staged, so
            // the TMA reads box c while the warpgroup stages box c + 1
#pragma unroll
            for (int c = 0; c < (OF16 ? 0 : D / 32); ++c) {
                constexpr int GROUP = C::TILE_BYTES / 16384;           // boxes in one Q tile
                const int slot = own_q ? c % GROUP : c;
                if (own_q && c > 0 && c % GROUP == 0) {                // the group's stores have read it
                    if (store) bulk_wait_read_all();
                    asm volatile("bar.sync %0, 128;" ::"r"(1 + t) : "memory");
                }
                if (ok) {
                    uint32_t o[32];
                    if (t_iters > 0) {
                        tmem_ld32(o_addr + c * 32, o);
                        tmem_ld_wait();
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = 0u;
                    }
#pragma unroll
                    for (int q4 = 0; q4 < 8; ++q4)
                        *reinterpret_cast<float4 *>(st + slot * 16384 + r * 128 + ((q4 ^ (r & 7)) << 4)) =
                            make_float4(__uint_as_float(o[4 * q4]) * inv, __uint_as_float(o[4 * q4 + 1]) * inv,
                                        __uint_as_float(o[4 * q4 + 2]) * inv, __uint_as_float(o[4 * q4 + 3]) * inv);
                }
                fence_proxy_async_smem();
                asm volatile("bar.sync %0, 128;" ::"r"(1 + t) : "memory");   // box c of this tile is staged
                if (store) {
                    tma_store_4d(&tmO, st + slot * 16384, c * 32, g * a.G, qt * a.tok_per_tile, b);
                    bulk_commit();
                }
            }
            if (store) bulk_wait_read_all();   // shared memory must stay valid until the stores have read it
        } else {
            // O rows are staged in the (now idle) Q tiles + K/V ring, padded by
            // 16 B per row, then written back as whole rows with 16 B per lane
            // (D/4 lanes per row), so every store fills complete 32 B sectors.
            constexpr int OP = D + 4;                               // staged row pitch (floats)
            static_assert(NQT * 128 * OP * 4 <= C::BAR_OFF, "O staging overlaps the barriers");
            float *stage = reinterpret_cast<float *>(smem + C::Q_OFF) + t * 128 * OP;
            if (ok) {
                tc_fence_after();
                if constexpr (C::ROWSUM) {
                    if (t_iters > 0) {
                        l_run = __uint_as_float(tmem_ld1(o_addr + D));
                        tmem_ld_wait();
                    }
                }
                const float inv = l_run == 0.0f ? 0.0f : 1.0f / l_run;
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
                    uint32_t o[32];
                    if (t_iters > 0) {
                        tmem_ld32(o_addr + c * 32, o);
                        tmem_ld_wait();
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = 0u;
                    }
#pragma unroll
                    for (int i = 0; i < 32; i += 4)
                        *reinterpret_cast<float4 *>(stage + r * OP + c * 32 + i) =
                            make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                                        __uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
                }
            }
            asm volatile("bar.sync %0, 128;" ::"r"(1 + t) : "memory");   // this warpgroup's rows are staged
            if (__all_sync(0xffffffffu, ok)) {
                constexpr int LPR = D / 4;                         // lanes per row (16 B each)
                constexpr int RPP = 128 / LPR;                     // rows per pass of the warpgroup
                const int c4 = r % LPR;
                int rr = r / LPR;
                if (qt < a.n_tiles_q && rr < rows_per_tile) {
                    // row rr = token-in-tile * G + head-in-group; advanced by RPP rows per
                    // pass with one division up front instead of one per row
                    int tk = qt * a.tok_per_tile + rr / a.G, hl = rr % a.G;
                    const int tk_step = RPP / a.G, hl_step = RPP % a.G;
                    const char *base = a.dst + (long long)b * a.d_nb3 + (long long)g * a.G * a.d_nb1 + c4 * 16;
                    for (; rr < rows_per_tile && tk < a.n_q; rr += RPP) {
                        *reinterpret_cast<float4 *>(const_cast<char *>(base) + (long long)tk * a.d_nb2 +
                                                    (long long)hl * a.d_nb1) =
                            *reinterpret_cast<const float4 *>(stage + rr * OP + c4 * 4);
                        hl += hl_step;
                        tk += tk_step;
                        if (hl >= a.G) {
                            hl -= a.G;
                            ++tk;
                        }
                    }
                }
            }
        }
    } else {
        if (NQT == 2) setmaxnreg_dec<C::REG_PRODUCER>();
        if (warp == C::TMA_WARP) {
            // =================== TMA producer =================================
            if (lane == 0) {
                const int bkv = b / a.kv_bdiv;
                if (a.q_tma) {
                    // the Q tiles first: box = 64 columns x G heads x tok_per_tile
                    // tokens, i.e. the tile's 128 rows (token * G + head)
                    mbar_arrive_expect_tx(q_full, NQT * C::TILE_BYTES);
#pragma unroll
                    for (int t = 0; t < NQT; ++t)
#pragma unroll
                        for (int sub = 0; sub < C::SUB; ++sub)
                            tma_load_4d(smem + C::Q_OFF + t * C::TILE_BYTES + sub * 16384, &tmQ, q_full, sub * 64,
                                        g * a.G, (qt0 + t) * a.tok_per_tile, b);
                }
                int issued = 0;
                for (int it = 0; it < n_iter; ++it) {
                    const int st = it % C::STAGES;
                    if (it >= C::STAGES &&
                        !mbar_wait(&kv_empty[st], ((it / C::STAGES) - 1) & 1, a.err, VTX_KERR_KV)) break;
                    issued = it + 1;
                    const int y = (j_begin + it) * C::BN;
                    char *ks = smem + C::K_OFF + st * C::TILE_BYTES;
                    char *vs = smem + C::V_OFF + st * C::TILE_BYTES;
                    mbar_arrive_expect_tx(&kv_full[st], C::TILE_BYTES);
                    mbar_arrive_expect_tx(&v_full[st], C::TILE_BYTES);
#pragma unroll
                    for (int sub = 0; sub < C::SUB; ++sub)
                        tma_load_4d(ks + sub * 16384, &tmK, &kv_full[st], sub * 64, y, g, bkv);
#pragma unroll
                    for (int sub = 0; sub < C::SUB; ++sub)
                        tma_load_4d(vs + sub * 16384, &tmV, &v_full[st], sub * 64, y, g, bkv);
                }
                // Drain: the last STAGES loads must have landed before this CTA's
                // shared memory is released (already true unless a wait failed).
                for (int it = issued > C::STAGES ? issued - C::STAGES : 0; it < issued; ++it) {
                    const int st = it % C::STAGES;
                    mbar_wait(&kv_full[st], (it / C::STAGES) & 1, a.err, VTX_KERR_KV);
                    mbar_wait(&v_full[st], (it / C::STAGES) & 1, a.err, VTX_KERR_KV);
                }
            }
        } else if (warp == C::MMA_WARP) {
            // =================== MMA issuer ===================================
            // Descriptor words are built once; per MMA only the low word (start
            // address >> 4) moves by a compile-time offset, so the issuing
            // thread spends a few cycles per tcgen05.mma instead of rebuilding
            // 64-bit descriptors.
            if (n_iter > 0) {
                const uint32_t lead = elect_one();     // the warp stays converged
                constexpr uint32_t IDESC_QK = idesc_f16_f32(128, 128, 0, 0);
                constexpr uint32_t IDESC_PV = idesc_f16_f32(128, C::OC, 0, 1);
                constexpr uint32_t HI = (1024u >> 4) | (1u << 14) | (2u << 29);   // SBO 1024, v1, SW128
                const uint32_t sbase = smem_u32(smem);
                const uint32_t lo_q = ((sbase + C::Q_OFF) >> 4) | (1u << 16);          // LBO 16 B (K-major)
                const uint32_t lo_k = ((sbase + C::K_OFF) >> 4) | (1u << 16);
                const uint32_t lo_v = ((sbase + C::V_OFF) >> 4) | ((16384u >> 4) << 16); // LBO: next 64 cols
                constexpr uint32_t T16 = C::TILE_BYTES >> 4;
                bool good = __all_sync(0xffffffffu, mbar_wait(q_full, 0, a.err, VTX_KERR_Q));
                tc_fence_after();
                // S_t = Q_t K^T of the key tile in stage `kst`
                auto issue_qk = [&](int t, int kst) {
                    const uint32_t s_tm = tmem + C::s_col(t);
                    const uint32_t q_lo = lo_q + t * T16;
                    const uint32_t k_lo = lo_k + kst * T16;
                    mma_f16_ss_w(lead, s_tm, desc64(q_lo, HI), desc64(k_lo, HI), IDESC_QK, 0u);
#pragma unroll
                    for (int kk = 1; kk < D / 16; ++kk) {
                        const uint32_t ko = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
                        mma_f16_ss_w(lead, s_tm, desc64(q_lo + ko, HI), desc64(k_lo + ko, HI), IDESC_QK, 1u);
                    }
                    mma_commit_w(lead, &s_full[t]);
                };
                // O_t (+)= P_t V of the key tile in stage `vst`
                auto issue_pv = [&](int t, int vst, uint32_t acc) {
                    const uint32_t p_tm = tmem + C::p_col(t);
                    const uint32_t o_tm = tmem + C::o_col(t);
                    // ROWSUM: the leading-byte offset reaches the constant block after the V ring
                    const uint32_t v_lo = C::ROWSUM ? (((sbase + C::V_OFF) >> 4) + vst * T16) |
                                                          (((uint32_t)(C::ONES_OFF - C::V_OFF) / 16u - vst * T16) << 16)
                                                    : lo_v + vst * T16;
                    mma_f16_ts_w(lead, o_tm, p_tm, desc64(v_lo, HI), IDESC_PV, acc);
#pragma unroll
                    for (int kk = 1; kk < 8; ++kk)
                        mma_f16_ts_w(lead, o_tm, p_tm + kk * 8, desc64(v_lo + kk * (2048 >> 4), HI), IDESC_PV, 1u);
                };
                if constexpr (C::LA) {
                    // Issue order per key tile it: S(it+1) for every Q tile as soon
                    // as its softmax has copied S(it) out, then O += P(it) V(it).
                    if (good) good = __all_sync(0xffffffffu, mbar_wait(&kv_full[0], 0, a.err, VTX_KERR_KV));
                    tc_fence_after();
                    if (good) {
#pragma unroll
                        for (int t = 0; t < NQT; ++t) issue_qk(t, 0);
                    }
                    for (int it = 0; it < n_iter && good; ++it) {
                        const int st = it % C::STAGES;
                        if (it + 1 < n_iter) {
                            const int nst = (it + 1) % C::STAGES;
                            if (!__all_sync(0xffffffffu, mbar_wait(&kv_full[nst], ((it + 1) / C::STAGES) & 1, a.err, VTX_KERR_KV))) {
                                good = false;
                                break;
                            }
#pragma unroll
                            for (int t = 0; t < NQT; ++t) {
                                if (!__all_sync(0xffffffffu, mbar_wait(&s_free[t], it & 1, a.err, VTX_KERR_S))) {
                                    good = false;
                                    break;
                                }
                                tc_fence_after();
                                issue_qk(t, nst);
                            }
                            if (!good) break;
                        }
                        if (!__all_sync(0xffffffffu, mbar_wait(&v_full[st], (it / C::STAGES) & 1, a.err, VTX_KERR_KV))) {
                            good = false;
                            break;
                        }
#pragma unroll
                        for (int t = 0; t < NQT; ++t) {
                            if (!__all_sync(0xffffffffu, mbar_wait(&p_full[t], it & 1, a.err, VTX_KERR_P))) {
                                good = false;
                                break;
                            }
                            tc_fence_after();
                            issue_pv(t, st, it > 0 ? 1u : 0u);
                            mma_commit_w(lead, &pv_done[t]);
                        }
                        if (!good) break;
                        mma_commit_w(lead, &kv_empty[st]);
                    }
                }
                uint32_t o_done = 0;                   // EARLY_O: tiles whose o_tile was committed
                for (int it = 0; !C::LA && it <= n_iter && good; ++it) {
                    const int st = it % C::STAGES;
                    const int pst = (it + C::STAGES - 1) % C::STAGES;
                    // V of the tile whose P V is due (it - 1), K of the one whose
                    // S is due (it): each waited for just before its first use
                    bool v_ready = it == 0, k_ready = it == n_iter;
#pragma unroll
                    for (int t = 0; t < NQT; ++t) {
                        int t_lo, t_hi;
                        tile_iters(t, t_lo, t_hi);
                        const int pi = it - 1;                 // the key tile whose P V is due
                        if (pi >= t_lo && pi < t_hi) {
                            if (!v_ready) {
                                if (!__all_sync(0xffffffffu,
                                                mbar_wait(&v_full[pst], (pi / C::STAGES) & 1, a.err, VTX_KERR_KV))) {
                                    good = false;
                                    break;
                                }
                                v_ready = true;
                            }
                            if (!__all_sync(0xffffffffu, mbar_wait(&p_full[t], (pi - t_lo) & 1, a.err, VTX_KERR_P))) {
                                good = false;
                                break;
                            }
                            tc_fence_after();
                            issue_pv(t, pst, pi > t_lo ? 1u : 0u);
                            if (EARLY_O && pi == t_hi - 1) {   // tile t's O is final
                                mma_commit_w(lead, &o_tile[t]);
                                o_done |= 1u << t;
                            }
                        }
                        if (it >= t_lo && it < t_hi) {
                            if (!k_ready) {
                                if (!__all_sync(0xffffffffu,
                                                mbar_wait(&kv_full[st], (it / C::STAGES) & 1, a.err, VTX_KERR_KV))) {
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
                    if (it > 0) mma_commit_w(lead, &kv_empty[pst]);
                }
                if (EARLY_O) {                         // a failed wait above: release the write-back
#pragma unroll
                    for (int t = 0; t < NQT; ++t)
                        if (!((o_done >> t) & 1u)) mma_commit_w(lead, &o_tile[t]);
                }
                mma_commit_w(lead, o_full);
                // every MMA of this CTA must be retired before TMEM is released
                mbar_wait(o_full, 0, a.err, VTX_KERR_O);
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
