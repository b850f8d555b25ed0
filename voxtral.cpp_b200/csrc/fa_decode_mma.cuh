// fa_decode_mma.cuh — HBM-streaming decode attention for sm_100a (F16 KV).
//
// The decode node of src/voxtral.cpp:1802 (n_tokens = 1, mask = NULL; one
// decode step per stream) reads every K/V row of the cache once and does ~4
// FLOP per byte, so it is bound by HBM.  Design:
//
//   * one WARP per work item (stream, KV head, key split); 4 warps per CTA on
//     adjacent KV heads of the same tokens, so a CTA reads contiguous 1 KB of
//     each token row of the [kv_dim, n_ctx] cache;
//   * each warp streams its rows through a private STAGES-deep ring in shared
//     memory: every lane issues one cp.async.bulk of one 256-byte K or V row
//     (16 keys x K+V per stage), completion counted by an mbarrier, rows
//     stored at a 16-byte padded pitch so ldmatrix reads are conflict-free;
//   * no CTA-wide barrier anywhere: warps run independently and ~128 KB per
//     SM are in flight;
//   * the G = Hq/Hkv query rows of the GQA group are the M operand of
//     mma.sync m16n8k16 (rows G..15 zero): S = Q K^T per 8 keys, the S
//     accumulator fragment becomes the f16 A fragment of O += P V directly,
//     so a 16-key step is ~100 instructions instead of ~900 on CUDA cores.
//
// Numerics follow ggml's CPU kernel for an F16 cache: Q rounded to half, f32
// accumulation of Q.K; P rounded to half for the PV product (ggml keeps the
// whole V accumulator in half), O accumulated in f32; softmax in the log2
// domain with lazy rescaling (only when the running max grows by > 2^8).
// Partials (m, l, o) use the layout of fa_combine_kernel.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "vtx_ptx.cuh"
#include "fa_splitkv.cuh"

namespace vtx {

template <int D> struct DecodeCfg {
    static constexpr int KEYS = 16;                 // keys per stage
    static constexpr int STAGES = 3;
    static constexpr int WARPS = 4;                 // work items per CTA
    static constexpr int ROW = D * 2;               // bytes per K or V row
    static constexpr int PITCH = ROW + 16;          // padded row pitch in shared memory
    static constexpr int STAGE_BYTES = 2 * KEYS * PITCH;
    static constexpr int WARP_BYTES = STAGES * STAGE_BYTES;
    static constexpr int SMEM = WARPS * WARP_BYTES + WARPS * STAGES * 8 + 64;
};

__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
// D = A (16x16 f16, row) * B (16x8 f16, col) + C, f32 accumulate
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One step of 16 keys for one warp, in two halves so that K and V can share
// one staging tile.  decode_scores: S = Q K^T (rows = the G query heads of the
// group, keys in two 8-wide halves), online softmax of this lane's row (lazy
// rescale of O), P packed as the A fragment of the PV product.  decode_pv:
// O += P V.  ks / vs: 16 rows of D halves at byte pitch PITCH (rows >= n hold
// zeros); qa: the Q A-fragments; cx = scale * log2(e).
// Online softmax of this lane's row of S (16 rows x 16 keys held as two 16x8
// accumulators s0 = keys 0-7, s1 = keys 8-15): lazy rescale of O, P packed
// as the A fragment of the PV product.
template <int D>
__device__ __forceinline__ void decode_softmax(const float (&s0)[4], const float (&s1)[4], int n, float cx,
                                               float (&o)[D / 8][4], float &m_run, float &l_part, int lane,
                                               uint32_t (&pa)[4])
{
    constexpr int NB = D / 8;
    // this lane's row: keys 2(l%4)+{0,1} (s0) and 8+2(l%4)+{0,1} (s1)
    const int kk = 2 * (lane & 3);
    float x[4] = {s0[0] * cx, s0[1] * cx, s1[0] * cx, s1[1] * cx};
    if (n < 16) {
        if (kk >= n) x[0] = -INFINITY;
        if (kk + 1 >= n) x[1] = -INFINITY;
        if (kk + 8 >= n) x[2] = -INFINITY;
        if (kk + 9 >= n) x[3] = -INFINITY;
    }
    float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    if (mx > m_run + 8.0f) {                        // lazy rescale, uniform within the quad
        const float alpha = m_run == -INFINITY ? 0.f : ex2(m_run - mx);
        m_run = mx;
        l_part *= alpha;
#pragma unroll
        for (int i = 0; i < NB; ++i) { o[i][0] *= alpha; o[i][1] *= alpha; }
    }
    const float mu = m_run == -INFINITY ? 0.f : m_run;
    const float p0 = ex2(x[0] - mu), p1 = ex2(x[1] - mu), p2 = ex2(x[2] - mu), p3 = ex2(x[3] - mu);
    l_part += (p0 + p1) + (p2 + p3);
    // P as the A fragment of the PV product (rows 8..15 zero)
    pa[0] = pack_half2(p0, p1);
    pa[1] = 0u;
    pa[2] = pack_half2(p2, p3);
    pa[3] = 0u;
}

// S = Q K^T for 16 keys (rows = the G query heads of the group) from K rows in
// shared memory (ldmatrix), then decode_softmax.  Even and odd dim chunks
// accumulate in separate chains (half the dependent-MMA latency).
template <int D, int PITCH>
__device__ __forceinline__ void decode_scores(const char *ks, int n, const uint32_t (&qa)[D / 16][4], float cx,
                                              float (&o)[D / 8][4], float &m_run, float &l_part, int lane,
                                              uint32_t (&pa)[4])
{
    constexpr int KC = D / 16;
    const int lrow = lane & 7, lmat = lane >> 3;    // ldmatrix: lane -> (row within 8x8, matrix)
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
    float e0[4] = {0.f, 0.f, 0.f, 0.f}, e1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kc = 0; kc < KC; kc += 2) {
        // matrices: keys 0-7 x dims [16kc, +8), [+8, +16), [+16, +24), [+24, +32)
        uint32_t bk[4], bk2[4];
        ldsm_x4(bk, ks + lrow * PITCH + (kc * 16 + lmat * 8) * 2);
        ldsm_x4(bk2, ks + (8 + lrow) * PITCH + (kc * 16 + lmat * 8) * 2);
        mma16816(s0, qa[kc], bk[0], bk[1]);
        mma16816(s1, qa[kc], bk2[0], bk2[1]);
        mma16816(e0, qa[kc + 1], bk[2], bk[3]);
        mma16816(e1, qa[kc + 1], bk2[2], bk2[3]);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        s0[i] += e0[i];
        s1[i] += e1[i];
    }
    decode_softmax<D>(s0, s1, n, cx, o, m_run, l_part, lane, pa);
}

template <int D, int PITCH>
__device__ __forceinline__ void decode_pv(const char *vs, const uint32_t (&pa)[4], float (&o)[D / 8][4], int lane)
{
    constexpr int NB = D / 8;
    const int lrow = lane & 7, lmat = lane >> 3;
    // O (16 x D) += P (16 x 16 keys) V (16 keys x D): B fragments by ldmatrix.trans
#pragma unroll
    for (int nb = 0; nb < NB; nb += 2) {
        // matrices: keys 0-7 / 8-15 x dims [8nb, +8), [8nb+8, +16)
        uint32_t bv[4];
        ldsm_x4_t(bv, vs + ((lmat & 1) * 8 + lrow) * PITCH + (nb * 8 + (lmat >> 1) * 8) * 2);
        mma16816(o[nb], pa, bv[0], bv[1]);
        mma16816(o[nb + 1], pa, bv[2], bv[3]);
    }
}

template <int D, int PITCH>
__device__ __forceinline__ void decode_tile(const char *ks, const char *vs, int n, const uint32_t (&qa)[D / 16][4],
                                            float cx, float (&o)[D / 8][4], float &m_run, float &l_part, int lane)
{
    uint32_t pa[4];
    decode_scores<D, PITCH>(ks, n, qa, cx, o, m_run, l_part, lane, pa);
    decode_pv<D, PITCH>(vs, pa, o, lane);
}

// Writes one lane's share of a (G x D) result: the final normalised rows
// (write_final) or the split's partial (O, m, l) in the combine layout.
template <int D>
__device__ __forceinline__ void decode_store(const SplitArgs &a, int b, int g, int sp, const float (&o)[D / 8][4],
                                             float m_run, float l_part, int lane)
{
    constexpr int NB = D / 8;
    const int qrow = lane >> 2;
    float l = l_part;
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (qrow < a.G) {
        const int h = g * a.G + qrow;
        const int kk = 2 * (lane & 3);              // this lane's output columns within each 8-block
        const long long work = ((long long)b * a.Hkv + g) * a.n_splits + sp;   // n_qtiles = n_hchunks = 1
        if (a.write_final) {
            float *out = reinterpret_cast<float *>(a.dst + (long long)h * a.d_nb1 + (long long)b * a.d_nb3);
            const float inv = l == 0.f ? 0.f : 1.f / l;
#pragma unroll
            for (int nb = 0; nb < NB; ++nb)
                *reinterpret_cast<float2 *>(out + nb * 8 + kk) = make_float2(o[nb][0] * inv, o[nb][1] * inv);
        } else {
            float *po = a.part_o + (work * 4 + qrow) * D;
#pragma unroll
            for (int nb = 0; nb < NB; ++nb)
                *reinterpret_cast<float2 *>(po + nb * 8 + kk) = make_float2(o[nb][0], o[nb][1]);
            if ((lane & 3) == 0) {
                a.part_ml[(work * 4 + qrow) * 2 + 0] = m_run;
                a.part_ml[(work * 4 + qrow) * 2 + 1] = l;
            }
        }
    }
}

template <int D>
__global__ void __launch_bounds__(128, 2)
fa_decode_mma_kernel(const SplitArgs a, int n_items)
{
    // With a.fresh only q and one row per stream come from the kernel launched
    // just before: the ring fills before waiting for it (see issue() and Q).
    const bool early = a.fresh != nullptr;
    if (!early) grid_dep_wait();
    grid_dep_launch();
    using C = DecodeCfg<D>;
    constexpr int KC = D / 16;                      // 16-wide chunks of the head dim
    extern __shared__ __align__(128) char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    char *ring = smem + warp * C::WARP_BYTES;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::WARPS * C::WARP_BYTES) + warp * C::STAGES;

    // work item: consecutive warps = consecutive KV heads of the same tokens
    const int item = blockIdx.x * C::WARPS + warp;
    const bool active = item < n_items;
    const int g = item % a.Hkv;
    const int sp = (item / a.Hkv) % a.n_splits;
    const int b = item / (a.Hkv * a.n_splits);

    int kv_len = a.n_kv;
    const char *kbase = nullptr, *vbase = nullptr;
    if (active) {
        if (a.k_ptrs) {
            kv_len = a.kv_len[b];
            kbase = static_cast<const char *>(a.k_ptrs[b]);
            vbase = static_cast<const char *>(a.v_ptrs[b]);
        } else {
            kbase = a.k + (long long)(b / a.k_bdiv) * a.k_nb3;
            vbase = a.v + (long long)(b / a.v_bdiv) * a.v_nb3;
        }
        kbase += (long long)g * a.k_nb2;
        vbase += (long long)g * a.v_nb2;
    }
    const int kb = sp * a.chunk;
    const int ke = min(kb + a.chunk, kv_len);
    // splits past this stream's length are not read by the combine kernel
    if (!active || (a.k_ptrs && sp > 0 && kb >= kv_len)) return;
    const bool misaligned = ((reinterpret_cast<uintptr_t>(kbase) | reinterpret_cast<uintptr_t>(vbase) |
                              (uintptr_t)a.k_nb1 | (uintptr_t)a.v_nb1) & 15) != 0;
    if (misaligned && lane == 0 && a.err) atomicCAS(a.err, 0, 7);
    const int ntiles = (ke > kb && !misaligned) ? (ke - kb + C::KEYS - 1) / C::KEYS : 0;

    if (lane < C::STAGES) mbar_init(&full[lane], 1);
    __syncwarp();
    fence_mbar_init();
    __syncwarp();
    const int fresh = early && a.k_ptrs ? a.fresh[b] : -1;   // row the preceding kernel writes
    bool waited = !early;
    auto dep_wait = [&]() {                          // warp-uniform
        if (!waited) {
            grid_dep_wait();
            waited = true;
        }
    };

    // ---- loader: lane l copies K row l (l < 16) or V row l-16 of a stage ----
    auto issue = [&](int t) {
        if (t >= ntiles) return;
        char *st = ring + (t % C::STAGES) * C::STAGE_BYTES;
        const int k0 = kb + t * C::KEYS;
        const int n = min(C::KEYS, ke - k0);
        if (fresh >= k0 && fresh < k0 + n) dep_wait();   // this stage holds the fresh row
        fence_proxy_async_smem();                    // our generic reads of this stage come first
        if (lane == 0) mbar_arrive_expect_tx(&full[t % C::STAGES], (uint32_t)(2 * n * C::ROW));
        __syncwarp();
        const int r = lane & 15;
        if (r >= n) {
            // rows past the key range are never loaded: zero them so P = 0
            // multiplies zeros, not stale shared memory (0 * NaN = NaN)
            uint4 *z = reinterpret_cast<uint4 *>(st + (lane < 16 ? r : C::KEYS + r) * C::PITCH);
#pragma unroll
            for (int i = 0; i < C::ROW / 16; ++i) z[i] = make_uint4(0u, 0u, 0u, 0u);
        }
        if (r < n) {
            if (lane < 16)
                bulk_g2s(st + r * C::PITCH, kbase + (long long)(k0 + r) * a.k_nb1, C::ROW, &full[t % C::STAGES]);
            else
                bulk_g2s(st + (C::KEYS + r) * C::PITCH, vbase + (long long)(k0 + r) * a.v_nb1, C::ROW,
                         &full[t % C::STAGES]);
        }
        __syncwarp();                                // zero rows visible to the whole warp
    };
#pragma unroll
    for (int t = 0; t < C::STAGES; ++t) issue(t);

    // ---- Q rows of the group as the A fragment (rows >= G are zero) ---------
    // A fragment of m16n8k16: a0 (row l/4, col 2(l%4)), a1 (row+8), a2 (col+8), a3 (row+8, col+8)
    const int qrow = lane >> 2;
    uint32_t qa[KC][4];
    dep_wait();                                      // q is written by the preceding kernel
    {
        const bool rq = qrow < a.G;
        const char *qp = a.q + (long long)(g * a.G + (rq ? qrow : 0)) * a.q_nb2 + (long long)b * a.q_nb3;
#pragma unroll
        for (int kc = 0; kc < KC; ++kc) {
            const int c = kc * 16 + 2 * (lane & 3);
            float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f;
            if (rq) {
                if (a.q_f16) {
                    const __half *hq = reinterpret_cast<const __half *>(qp);
                    x0 = __half2float(hq[c]); x1 = __half2float(hq[c + 1]);
                    x2 = __half2float(hq[c + 8]); x3 = __half2float(hq[c + 9]);
                } else {
                    const float *fq = reinterpret_cast<const float *>(qp);
                    x0 = fq[c]; x1 = fq[c + 1]; x2 = fq[c + 8]; x3 = fq[c + 9];
                }
            }
            qa[kc][0] = pack_half2(x0, x1);        // ggml rounds Q to half for an F16 K
            qa[kc][1] = 0u;
            qa[kc][2] = pack_half2(x2, x3);
            qa[kc][3] = 0u;
        }
    }

    // ---- stream the keys ------------------------------------------------------
    constexpr int NB = D / 8;                       // n-blocks of 8 output dims
    float o[NB][4];
#pragma unroll
    for (int i = 0; i < NB; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run = -INFINITY, l_part = 0.f;         // this lane's row (qrow), partial sum
    const float cx = a.qk_scale * kLog2e;
    bool ok = true;
    int t_done = 0;

    for (int t = 0; t < ntiles && ok; ++t) {
        const int stg = t % C::STAGES;
        ok = __all_sync(0xffffffffu, mbar_wait(&full[stg], (t / C::STAGES) & 1, a.err, VTX_KERR_KV));
        if (!ok) break;
        const char *ks = ring + stg * C::STAGE_BYTES;
        const char *vs = ks + C::KEYS * C::PITCH;
        const int k0 = kb + t * C::KEYS;
        decode_tile<D, C::PITCH>(ks, vs, min(C::KEYS, ke - k0), qa, cx, o, m_run, l_part, lane);
        __syncwarp();                               // every lane has read this stage
        issue(t + C::STAGES);
        t_done = t + 1;
    }
    // after a failed wait: let this warp's copies still in flight land (bounded)
    for (int t = t_done; t < min(ntiles, t_done + C::STAGES); ++t)
        mbar_wait(&full[t % C::STAGES], (t / C::STAGES) & 1, nullptr, 0);

    // ---- write the partial (or the final row) ---------------------------------
    decode_store<D>(a, b, g, sp, o, m_run, l_part, lane);
}

}  // namespace vtx
