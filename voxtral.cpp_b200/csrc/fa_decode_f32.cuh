// fa_decode_f32.cuh — HBM-streaming decode attention over the reference's
// own F32 KV cache (sm_100a).
//
// voxtral.cpp keeps its decoder cache in F32 (src/voxtral.cpp:1126-1136),
// and ggml's CPU kernel then computes the decode node (src/voxtral.cpp:1802,
// n_tokens = 1) entirely in f32: Q . K in f32 (ggml_vec_dot_f32), the V
// accumulator in f32 (ggml_vec_mad_f32).  This kernel does the same f32
// arithmetic on CUDA cores, streaming the rows the way the F16 kernel does:
//
//   * one warp per work item (stream, KV head, key split), 4 warps per CTA on
//     adjacent KV heads of the same tokens;
//   * a private STAGES-deep ring per warp: a lane bulk-copies one K or V row
//     (D floats) of an 8-key stage (16 keys for D = 64), completion counted
//     by an mbarrier; 96 KB per CTA, two CTAs per SM;
//   * lane (h, c) = (query head h of the GQA group, chunk lane c of 8) holds
//     Q[h] and O[h] for D / 8 dims in registers: the float4 groups c, c + 8,
//     c + 16, ... of the row, so one 16-byte shared load of the 8 chunk lanes
//     reads 128 contiguous bytes (no bank conflicts); the 4 head lanes of a
//     chunk lane read the same bytes (a broadcast).  Per stage a lane forms
//     its partial Q . K over its dims for the stage's keys, reduces them over
//     the 8 chunk lanes (butterfly shuffles), runs the online softmax of head
//     h (log2 domain, lazy rescale past a 2^8 jump of the running max) and
//     adds P V for its dims.  The f32 dot products run as two chains per key
//     (a different summation order from ggml's vector loop, within f32
//     rounding of it).
// Partials (m, l, o) use fa_combine_kernel's layout.
#pragma once
#include <cstdint>
#include "vtx_ptx.cuh"
#include "fa_splitkv.cuh"
#include "fa_decode_mma.cuh"

namespace vtx {

template <int D> struct DecodeF32Cfg {
    static constexpr int KEYS = D == 64 ? 16 : 8;   // keys per stage (one K and one V row per lane)
    static constexpr int STAGES = 3;
    static constexpr int WARPS = 4;                 // work items per CTA
    static constexpr int ROW = D * 4;               // bytes per K or V row
    static constexpr int STAGE_BYTES = 2 * KEYS * ROW;
    static constexpr int WARP_BYTES = STAGES * STAGE_BYTES;
    static constexpr int SMEM = WARPS * WARP_BYTES + WARPS * STAGES * 8 + 64;
    static constexpr int DC = D / 8;                // dims per chunk lane
};

template <int D>
__global__ void __launch_bounds__(128, 2)
fa_decode_f32_kernel(const SplitArgs a, int n_items)
{
    // With a.fresh only q and one row per stream come from the kernel launched
    // just before: the ring fills before waiting for it (see issue() and Q).
    const bool early = a.fresh != nullptr;
    if (!early) grid_dep_wait();
    grid_dep_launch();
    using C = DecodeF32Cfg<D>;
    constexpr int DC = C::DC;
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

    // ---- loader: lane l copies K row l (l < KEYS) or V row l - KEYS of a stage ----
    auto issue = [&](int t) {
        if (t >= ntiles) return;
        char *st = ring + (t % C::STAGES) * C::STAGE_BYTES;
        const int k0 = kb + t * C::KEYS;
        const int n = min(C::KEYS, ke - k0);
        if (fresh >= k0 && fresh < k0 + n) dep_wait();   // this stage holds the fresh row
        fence_proxy_async_smem();                    // our generic reads of this stage come first
        if (lane == 0) mbar_arrive_expect_tx(&full[t % C::STAGES], (uint32_t)(2 * n * C::ROW));
        __syncwarp();
        const int r = lane % C::KEYS;                // lanes [0, KEYS): K rows, [KEYS, 2 KEYS): V rows
        const bool isk = lane < C::KEYS, mine = lane < 2 * C::KEYS;
        if (mine && r >= n) {
            // rows past the key range are never loaded: zero them so P = 0
            // multiplies zeros, not stale shared memory (0 * NaN = NaN)
            uint4 *z = reinterpret_cast<uint4 *>(st + (isk ? r : C::KEYS + r) * C::ROW);
#pragma unroll
            for (int i = 0; i < C::ROW / 16; ++i) z[i] = make_uint4(0u, 0u, 0u, 0u);
        }
        if (mine && r < n) {
            if (isk)
                bulk_g2s(st + r * C::ROW, kbase + (long long)(k0 + r) * a.k_nb1, C::ROW, &full[t % C::STAGES]);
            else
                bulk_g2s(st + (C::KEYS + r) * C::ROW, vbase + (long long)(k0 + r) * a.v_nb1, C::ROW,
                         &full[t % C::STAGES]);
        }
        __syncwarp();                                // zero rows visible to the whole warp
    };
#pragma unroll
    for (int t = 0; t < C::STAGES; ++t) issue(t);

    // ---- Q: lane (h, c) holds dims 32 i + 4 c + e (i < DC / 4, e < 4) of head h --
    const int h = lane >> 3, c = lane & 7;
    const bool hq = h < a.G;
    float q[DC];
    dep_wait();                                      // q is written by the preceding kernel
    {
        const char *qp = a.q + (long long)(g * a.G + (hq ? h : 0)) * a.q_nb2 + (long long)b * a.q_nb3;
#pragma unroll
        for (int i = 0; i < DC; ++i) {
            float x = 0.f;
            const int d = (i >> 2) * 32 + c * 4 + (i & 3);
            if (hq) x = a.q_f16 ? __half2float(reinterpret_cast<const __half *>(qp)[d])
                                : reinterpret_cast<const float *>(qp)[d];
            q[i] = x;
        }
    }

    float o[DC];
#pragma unroll
    for (int i = 0; i < DC; ++i) o[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;            // head h's state (the same in its 8 lanes)
    const float cx = a.qk_scale * kLog2e;
    bool ok = true;
    int t_done = 0;

    for (int t = 0; t < ntiles && ok; ++t) {
        const int stg = t % C::STAGES;
        ok = __all_sync(0xffffffffu, mbar_wait(&full[stg], (t / C::STAGES) & 1, a.err, VTX_KERR_KV));
        if (!ok) break;
        const char *ks = ring + stg * C::STAGE_BYTES;
        const char *vs = ks + C::KEYS * C::ROW;
        const int n = min(C::KEYS, ke - (kb + t * C::KEYS));
        // partial scores over this lane's dims, then the sum over the 8 chunks
        float s[C::KEYS];
#pragma unroll
        for (int j = 0; j < C::KEYS; ++j) {
            const float4 *kr = reinterpret_cast<const float4 *>(ks + j * C::ROW) + c;
            float acc0 = 0.f, acc1 = 0.f;                // two chains per key
#pragma unroll
            for (int i = 0; i < DC / 4; ++i) {
                const float4 k4 = kr[8 * i];
                acc0 = fmaf(q[4 * i], k4.x, acc0);
                acc1 = fmaf(q[4 * i + 1], k4.y, acc1);
                acc0 = fmaf(q[4 * i + 2], k4.z, acc0);
                acc1 = fmaf(q[4 * i + 3], k4.w, acc1);
            }
            s[j] = acc0 + acc1;
        }
#pragma unroll
        for (int x = 1; x < 8; x <<= 1)
#pragma unroll
            for (int j = 0; j < C::KEYS; ++j) s[j] += __shfl_xor_sync(0xffffffffu, s[j], x);
        // online softmax of head h over the stage's keys (keys >= n masked)
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < C::KEYS; ++j) {
            s[j] = j < n ? s[j] * cx : -INFINITY;
            mx = fmaxf(mx, s[j]);
        }
        if (mx > m_run + 8.0f) {                     // lazy rescale: only on a 2^8 jump
            const float alpha = m_run == -INFINITY ? 0.f : ex2(m_run - mx);
            m_run = mx;
            l_run *= alpha;
#pragma unroll
            for (int i = 0; i < DC; ++i) o[i] *= alpha;
        }
        const float mu = m_run == -INFINITY ? 0.f : m_run;
#pragma unroll
        for (int j = 0; j < C::KEYS; ++j) {
            const float p = ex2(s[j] - mu);
            l_run += p;
            const float4 *vr = reinterpret_cast<const float4 *>(vs + j * C::ROW) + c;
#pragma unroll
            for (int i = 0; i < DC / 4; ++i) {
                const float4 v4 = vr[8 * i];
                o[4 * i] = fmaf(p, v4.x, o[4 * i]);
                o[4 * i + 1] = fmaf(p, v4.y, o[4 * i + 1]);
                o[4 * i + 2] = fmaf(p, v4.z, o[4 * i + 2]);
                o[4 * i + 3] = fmaf(p, v4.w, o[4 * i + 3]);
            }
        }
        __syncwarp();                               // every lane has read this stage
        issue(t + C::STAGES);
        t_done = t + 1;
    }
    // after a failed wait: let this warp's copies still in flight land (bounded)
    for (int t = t_done; t < min(ntiles, t_done + C::STAGES); ++t)
        mbar_wait(&full[t % C::STAGES], (t / C::STAGES) & 1, nullptr, 0);

    // ---- write the partial (or the final row) ---------------------------------
    if (!hq) return;
    if (a.write_final) {
        float *out = reinterpret_cast<float *>(a.dst + (long long)(g * a.G + h) * a.d_nb1 + (long long)b * a.d_nb3);
        const float inv = l_run == 0.f ? 0.f : 1.f / l_run;
#pragma unroll
        for (int i = 0; i < DC; ++i) out[(i >> 2) * 32 + c * 4 + (i & 3)] = o[i] * inv;
    } else {
        const long long work = ((long long)b * a.Hkv + g) * a.n_splits + sp;
        float4 *po = reinterpret_cast<float4 *>(a.part_o + (work * 4 + h) * D) + c;
#pragma unroll
        for (int i = 0; i < DC / 4; ++i) po[8 * i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        if (c == 0) {
            a.part_ml[(work * 4 + h) * 2 + 0] = m_run;
            a.part_ml[(work * 4 + h) * 2 + 1] = l_run;
        }
    }
}

}  // namespace vtx
