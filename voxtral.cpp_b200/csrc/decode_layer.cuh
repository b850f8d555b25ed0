// decode_layer.cuh — one decoder layer's attention step in one launch
// (sm_100a): RoPE of Q and K, the new K/V row into its cache ring slot, decode
// attention over the ring, and the merge of the key splits.
//
// Per decoded token and layer, voxtral.cpp runs ggml_rope_ext on Q and K, two
// ggml_cpy into the cache (src/voxtral.cpp:1744-1770) and the
// ggml_flash_attn_ext node (:1802) with n_tokens = 1.  At batch 1 that work is
// a few MB and the step is bound by the chain of dependent launches, not by
// HBM: append, attention and split merge as three kernels cost ~14 us per
// layer even for a 17-key cache.  Here all of it is one kernel:
//
//   grid      one CTA per (stream, KV head, key split); splits sized so that
//             one wave covers the GPU (one CTA per SM);
//   warps     W per CTA (8 for F16, 16 for Q8_0), each streaming every W-th
//             16-key tile of the CTA's key range through a private two-stage
//             ring (lane l bulk-copies K row l or V row l-16 of a tile; one
//             mbarrier per stage) -- issued before the dependency wait when
//             the caller allows it;
//   append    the warp whose tile holds the stream's new row (its ring slot)
//             rotates and converts the new K (and converts V) exactly as
//             vtx_kv_append does, writes the bytes to the cache and into its
//             ring stage in place of the copy;
//   compute   F16: mma.sync S = Q K^T / O += P V with the G query heads as
//             rows; Q8_0: int8 MMA S^T = K q8(Q) with ggml's block scales, V
//             dequantised to f16, O^T += V^T P^T (the arithmetic of the
//             streaming decode kernels for these cache types);
//   merge     the W warps' softmax states in shared memory, then, with more
//             than one split, a partial (O, m, l) per CTA, merged either
//             (CL) through distributed shared memory: the splits of a
//             (stream, KV head) are the CTAs of one thread-block cluster, two
//             cluster barriers, each CTA folding every split's partial for
//             its share of the rows -- for launches with few splits, whose
//             small clusters let the next layer's CTAs become resident early;
//             or through global memory: the last CTA of a (stream, KV head)
//             to arrive -- counted by one atomic increment that wraps to zero
//             on the last arrival, so the workspace needs zeroing once and
//             every call leaves it zeroed -- merges the partials and writes
//             ggml's F32 row.
//
// Numerics are those of the separate calls: Q rotated in f32 then rounded to
// half (F16 cache) or quantised per 32 values (Q8_0 cache), f32 scores and
// accumulators, P in half, softmax in the log2 domain with lazy rescaling.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "vtx_ptx.cuh"
#include "fa_decode_mma.cuh"
#include "fa_decode_q8.cuh"
#include "kv_append.cuh"

namespace vtx {

struct DecodeLayerArgs {
    int n_seq, Hq, Hkv, G;
    const float *q, *k, *v;                    // this step's projections, heads contiguous
    long long q_nb1, k_nb1, v_nb1;             // token strides (floats)
    const int *positions, *slots, *kv_len;
    const void *const *k_ptrs; const void *const *v_ptrs;
    long long cache_nb1;                       // bytes per cache row
    float theta_scale, cx;                     // RoPE step; scale * log2(e)
    float *dst; long long dst_nb1;             // token stride (floats), heads contiguous
    int n_splits;                              // key splits per (stream, head) in the grid (the most used)
    float *part_o, *part_ml;                   // split partials (n_splits > 1)
    unsigned *flags;                           // one arrival counter per (stream, KV head), zero between calls
    int early;                                 // ring rows and counters may be read before the dependency wait
    int *err;
};

template <int KVT> struct LayerCfg {
    // Warps per CTA and CTAs per SM.  Q8_0 tiles cost ~3x the instructions
    // of F16 ones (int8 fragments, block scales, V dequantised to half) with
    // long dependent chains: 16 warps per CTA (4 per scheduler) hide them;
    // F16 needs 8.  Measured on B200 (graph replay, 32/8 x 128, batch 1):
    // two CTAs per SM (8 / 4 warps, so the next layer's CTA overlaps this
    // one) wins below ~2000 Q8_0 keys and loses above (12.2 vs 12.0 us at
    // 7300 keys, 7.4 vs 6.6 us for F16 at 600 keys).
#ifndef VTX_LAYER_WQ8
#define VTX_LAYER_WQ8 16
#endif
#ifndef VTX_LAYER_WF16
#define VTX_LAYER_WF16 8
#endif
#ifndef VTX_LAYER_MINBQ8
#define VTX_LAYER_MINBQ8 1
#endif
#ifndef VTX_LAYER_MINBF16
#define VTX_LAYER_MINBF16 1
#endif
    static constexpr int W = KVT == 8 ? VTX_LAYER_WQ8 : VTX_LAYER_WF16;
    static constexpr int MINB = KVT == 8 ? VTX_LAYER_MINBQ8 : VTX_LAYER_MINBF16;
    static constexpr int D = 128, KEYS = 16, GMAX = 8;
    static constexpr int NT = W * 32;
    static constexpr int HB = KVT == 1 ? 256 : 136;            // one head's row in the cache
    static constexpr int ROWB = KVT == 1 ? 256 : 144;          // bytes per ring row copy (Q8_0: 16-B superset)
    static constexpr int PITCH = KVT == 1 ? 272 : 144;         // ring row pitch: conflict-free fragment loads
    static constexpr int STAGES = 2;
    static constexpr int STAGE_BYTES = 2 * KEYS * PITCH;       // K rows, then V rows
    static constexpr int RING = STAGES * STAGE_BYTES;          // per warp
    static constexpr int FPITCH = D * 2 + 16;                  // Q8_0: dequantised V tile row
    static constexpr int VTILE = KVT == 8 ? KEYS * FPITCH : 0; // per warp
    static constexpr int VT_OFF = W * RING;
    static constexpr int CS_OFF = VT_OFF + W * VTILE;          // the CTA's (cos, sin) table, 64 pairs
    static constexpr int BAR_OFF = CS_OFF + 64 * 8;
    static constexpr int QF_OFF = BAR_OFF + W * STAGES * 8;     // Q8_0: Q fragments [block][lane] (16 B)
    static constexpr int MISC_OFF = QF_OFF + (KVT == 8 ? D / 32 * 32 * 16 : 0);
    static constexpr int SMEM = MISC_OFF + 16;
    // after the key loop (rings idle): the warps' states, then the split merge
    // state rows padded so the warps' dumps are conflict-free (F16: float2
    // stores by 8 rows x 4 column pairs; Q8_0: 4-byte stores by 8 dims x 4 heads)
    static constexpr int SP = KVT == 1 ? D + 8 : D + 4;
    static constexpr int ST_ML = W * GMAX * SP * 4;            // [W][GMAX][SP] O, then [W][GMAX] (m, l)
    static constexpr int ST_F = ST_ML + W * GMAX * 8;          // [W][GMAX] merge factors, then [GMAX] 1/L or L
    static constexpr int GRP_OFF = ST_F + (W + 1) * GMAX * 4;  // split merge: [NT] float4 acc + (m, l)
    static_assert(GRP_OFF + NT * 24 <= W * RING, "merge buffers overlap the barriers");
    // cluster merge (CL): this split's O rows and (m, l) at GRP_OFF; at most
    // CLMAX splits (the portable cluster size)
    static constexpr int CLMAX = 8;
    static_assert(GRP_OFF + GMAX * D * 4 + GMAX * 8 <= W * RING, "cluster partial overlaps the barriers");
    static_assert(GRP_OFF % 16 == 0, "16-byte cluster loads of the partial");
};

// Arrival on a split counter: old value returned, the counter wraps to 0 on
// the arrival that finds it at `last` (atom.inc), with acquire-release
// semantics at gpu scope.
__device__ __forceinline__ unsigned arrive_inc_acq_rel(unsigned *p, unsigned last) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(last) : "memory");
    return old;
}

template <int KVT, bool CL>
__global__ void __launch_bounds__(LayerCfg<KVT>::NT, LayerCfg<KVT>::MINB)
fa_decode_layer_kernel(const DecodeLayerArgs a)
{
    using C = LayerCfg<KVT>;
    constexpr int D = C::D, KEYS = C::KEYS, W = C::W;
    if (!a.early) grid_dep_wait();
    grid_dep_launch();
    extern __shared__ __align__(128) char smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sp = blockIdx.x % a.n_splits;
    const int g = (blockIdx.x / a.n_splits) % a.Hkv;
    const int b = blockIdx.x / (a.n_splits * a.Hkv);

    // every per-stream word is loaded at once (independent round trips)
    const int kv_raw = a.kv_len[b];
    const int fresh = a.slots[b];
    const void *kp0 = a.k_ptrs[b], *vp0 = a.v_ptrs[b];
    const int pos = threadIdx.x < 64 ? a.positions[b] : 0;    // the RoPE position (table threads)
    // this stream's splits, from its key count: at most n_splits, at least one
    // 16-key tile per warp each (so short caches use fewer CTAs and merges),
    // and none up to two tiles per warp (measured: a Q8_0 cache of 500 keys
    // 6.4 us in one CTA per head vs 7.6 us in two with the merge)
    const int kv_len = max(0, kv_raw);
    const int tiles_b = (kv_len + KEYS - 1) / KEYS;
    const int s_eff = tiles_b <= 2 * W ? 1 : max(1, min(a.n_splits, (tiles_b + W - 1) / W));
    const int chunk = max(1, (tiles_b + s_eff - 1) / s_eff) * KEYS;
    const int nsp = max(1, (kv_len + chunk - 1) / chunk);
    const int kb = sp * chunk;
    const int ke = min(kb + chunk, kv_len);
    if (sp >= nsp) {                                           // past the stream's keys: not merged
        if constexpr (CL) {
            if (nsp > 1) {                                     // the cluster's two barriers, no partial
                cluster_arrive();
                cluster_wait();
                cluster_arrive();
                cluster_wait();
            }
        }
        return;
    }
    const char *kbase = static_cast<const char *>(kp0) + (long long)g * C::HB;
    const char *vbase = static_cast<const char *>(vp0) + (long long)g * C::HB;
    // Q8_0 rows (136 B) of odd heads sit 8 bytes past a 16-byte boundary: copy
    // the 144-byte superset from the boundary (the host requires an even head
    // count, so it stays inside the token row) and read the head from `off`
    const int off = (g * C::HB) & 15;
    const bool bad = ((reinterpret_cast<uintptr_t>(kp0) | reinterpret_cast<uintptr_t>(vp0) |
                       (uintptr_t)a.cache_nb1) & 15) != 0;
    if (bad && threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, 7);
    const char *ksrc = kbase - off, *vsrc = vbase - off;
    const int ntiles = (ke > kb && !bad) ? (ke - kb + KEYS - 1) / KEYS : 0;
    const int my_tiles = ntiles > warp ? (ntiles - warp + W - 1) / W : 0;   // tiles warp, warp + W, ...
    const int f_tile = (fresh >= kb && fresh < ke) ? (fresh - kb) / KEYS : -1;
    const int f_local = (f_tile >= 0 && f_tile % W == warp && !bad) ? f_tile / W : -1;

    char *ring = smem + warp * C::RING;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF) + warp * C::STAGES;
    const float2 *cs = reinterpret_cast<const float2 *>(smem + C::CS_OFF);
    if (lane < C::STAGES) mbar_init(&full[lane], 1);
    __syncwarp();
    fence_mbar_init();
    __syncwarp();

    // ---- the new row: K rotated, both converted, written to the cache and to
    //      ring row r of stage buffer st (the copy of that row is skipped)
    auto write_fresh = [&](char *st, int r) {
        const float4 kx = *reinterpret_cast<const float4 *>(a.k + (long long)b * a.k_nb1 + g * D + 4 * lane);
        const float4 vx = *reinterpret_cast<const float4 *>(a.v + (long long)b * a.v_nb1 + g * D + 4 * lane);
        float kr[4] = {kx.x, kx.y, kx.z, kx.w};
        const float vr[4] = {vx.x, vx.y, vx.z, vx.w};
        rope_pair(kr[0], kr[1], cs[2 * lane]);
        rope_pair(kr[2], kr[3], cs[2 * lane + 1]);
        char *kg = static_cast<char *>(const_cast<void *>(kp0)) + (long long)fresh * a.cache_nb1 + g * C::HB;
        char *vg = static_cast<char *>(const_cast<void *>(vp0)) + (long long)fresh * a.cache_nb1 + g * C::HB;
        char *ks = st + r * C::PITCH + off;
        char *vs = st + (KEYS + r) * C::PITCH + off;
        if constexpr (KVT == 1) {
            const uint2 kp = make_uint2(pack_half2(kr[0], kr[1]), pack_half2(kr[2], kr[3]));
            const uint2 vp = make_uint2(pack_half2(vr[0], vr[1]), pack_half2(vr[2], vr[3]));
            *reinterpret_cast<uint2 *>(kg + 8 * lane) = kp;
            *reinterpret_cast<uint2 *>(vg + 8 * lane) = vp;
            *reinterpret_cast<uint2 *>(ks + 8 * lane) = kp;
            *reinterpret_cast<uint2 *>(vs + 8 * lane) = vp;
        } else {
            store_q8_lane<4>(kr, kg, lane);
            store_q8_lane<4>(vr, vg, lane);
            store_q8_lane<4>(kr, ks, lane);
            store_q8_lane<4>(vr, vs, lane);
        }
    };

    // ---- ring: local tile i (= CTA tile warp + W i) into stage i % STAGES ----
    // The new row's copy is skipped; its bytes are written by write_fresh once
    // the (cos, sin) table exists (at once for tiles issued after it).
    bool table_ready = false;
    auto issue = [&](int i) {
        if (i >= my_tiles) return;
        const int t = warp + W * i;
        char *st = ring + (i % C::STAGES) * C::STAGE_BYTES;
        const int k0 = kb + t * KEYS;
        const int n = min(KEYS, ke - k0);
        const int rf = i == f_local ? fresh - k0 : -1;
        if (i >= C::STAGES) fence_proxy_async_smem();          // this warp's reads of the stage come first
        if (lane == 0) mbar_arrive_expect_tx(&full[i % C::STAGES], (uint32_t)(2 * (n - (rf >= 0)) * C::ROWB));
        __syncwarp();
        const int r = lane & 15;
        const bool isv = lane >= 16;
        if (r >= n) {
            if constexpr (KVT == 1) {                          // F16: P = 0 must multiply zeros, not stale data
                uint4 *z = reinterpret_cast<uint4 *>(st + (isv ? KEYS + r : r) * C::PITCH);
#pragma unroll
                for (int u = 0; u < C::ROWB / 16; ++u) z[u] = make_uint4(0u, 0u, 0u, 0u);
            }
        } else if (r != rf) {
            bulk_g2s(st + (isv ? KEYS + r : r) * C::PITCH, (isv ? vsrc : ksrc) + (long long)(k0 + r) * a.cache_nb1,
                     (uint32_t)C::ROWB, &full[i % C::STAGES]);
        }
        if (rf >= 0 && table_ready) write_fresh(st, rf);
        __syncwarp();
    };
#pragma unroll
    for (int i = 0; i < C::STAGES; ++i) issue(i);

    // ---- the CTA's (cos, sin) table: thread i < 64 runs the float angle
    //      recurrence i steps (ggml's rope cache), then one sincos (with early
    //      = 1 the positions, like the ring, come before the dependency wait)
    if (threadIdx.x < 64) {
        float th = (float)pos;
        for (int i = 0; i < (int)threadIdx.x; ++i) th *= a.theta_scale;
        reinterpret_cast<float2 *>(smem + C::CS_OFF)[threadIdx.x] = rope_cs(th);
    }

    // ---- dependency wait; Q of the group into registers (warps with tiles) ----
    if (a.early) grid_dep_wait();
    const float *qg = a.q + (long long)b * a.q_nb1 + (long long)g * a.G * D;
    constexpr int NB = D / 8, NJ = D / 16, KC = D / 16, NBLK = D / 32;
    // F16: every warp with tiles loads its A fragments (row l/4 = the query
    // head, columns 2(l%4)+{0,1} and +8 of every 16-column chunk).  Q8_0: warp
    // j < 4 loads block j (lane (r, c): head r's values 32j + 4c.. and
    // 32j + 16 + 4c..) and quantises it once for the CTA.
    float4 qx[KVT == 1 ? KC : 2];
    {
        const int qr = lane >> 2;
        const float *qp = qg + (qr < a.G ? qr : 0) * D;
        const bool rq = qr < a.G && (KVT == 1 ? my_tiles > 0 : warp < NBLK);
#pragma unroll
        for (int i = 0; i < (KVT == 1 ? KC : 2); ++i) {
            qx[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (rq) {
                if constexpr (KVT == 1) {
                    const int c = i * 16 + 2 * (lane & 3);
                    const float2 u = *reinterpret_cast<const float2 *>(qp + c);
                    const float2 w = *reinterpret_cast<const float2 *>(qp + c + 8);
                    qx[i] = make_float4(u.x, u.y, w.x, w.y);
                } else {
                    qx[i] = *reinterpret_cast<const float4 *>(qp + 32 * warp + 4 * (lane & 3) + 16 * i);
                }
            }
        }
    }
    __syncthreads();                                           // the table is complete
    table_ready = true;
    if (f_local >= 0 && f_local < C::STAGES) {                 // the new row's tile was issued above
        const int k0 = kb + (warp + W * f_local) * KEYS;
        write_fresh(ring + (f_local % C::STAGES) * C::STAGE_BYTES, fresh - k0);
        __syncwarp();
    }

    // ---- Q rotated, in the MMA operand layout ---------------------------------
    float o[KVT == 1 ? NB : NJ][4];
    float m_run[2] = {-INFINITY, -INFINITY}, l_part[2] = {0.f, 0.f};
    uint32_t qa[KVT == 1 ? KC : 1][4];
    uint32_t qb[KVT == 8 ? NBLK : 1][2];
    float dq[KVT == 8 ? NBLK : 1][2];
    if constexpr (KVT == 1) {
        // A fragment of m16n8k16 (rows >= G are zero), rounded to half as ggml
        // rounds Q for an F16 K
#pragma unroll
        for (int kc = 0; kc < KC; ++kc) {
            const int c = kc * 16 + 2 * (lane & 3);
            float4 x = qx[kc];
            rope_pair(x.x, x.y, cs[c / 2]);
            rope_pair(x.z, x.w, cs[c / 2 + 4]);
            qa[kc][0] = pack_half2(x.x, x.y);
            qa[kc][1] = 0u;
            qa[kc][2] = pack_half2(x.z, x.w);
            qa[kc][3] = 0u;
        }
#pragma unroll
        for (int i = 0; i < NB; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    } else {
        // s8 B fragment of block `warp`, quantised per 32 values as ggml's
        // from_float, shared through shared memory with the other warps
        uint4 *qf = reinterpret_cast<uint4 *>(smem + C::QF_OFF);
        if (warp < NBLK) {
            const int qc = lane & 3;
            float x[8];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int c = 32 * warp + 4 * qc + 16 * h;
                float4 u = qx[h];
                rope_pair(u.x, u.y, cs[c / 2]);
                rope_pair(u.z, u.w, cs[c / 2 + 1]);
                x[4 * h] = u.x; x[4 * h + 1] = u.y; x[4 * h + 2] = u.z; x[4 * h + 3] = u.w;
            }
            float amax = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(x[i]));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            const float d = __half2float(__float2half_rn(amax / 127.0f));
            const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
            uint32_t w[2] = {0u, 0u};
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i >> 2] |= ((uint32_t)__float2int_rn(x[i] * id) & 0xffu) << (8 * (i & 3));
            const float d0 = __shfl_sync(0xffffffffu, d, 8 * qc);          // head 2c
            const float d1 = __shfl_sync(0xffffffffu, d, 8 * qc + 4);      // head 2c + 1
            qf[warp * 32 + lane] = make_uint4(w[0], w[1], __float_as_uint(d0), __float_as_uint(d1));
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < NBLK; ++j) {
            const uint4 f = qf[j * 32 + lane];
            qb[j][0] = f.x;
            qb[j][1] = f.y;
            dq[j][0] = __uint_as_float(f.z);
            dq[j][1] = __uint_as_float(f.w);
        }
#pragma unroll
        for (int j = 0; j < NJ; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    }

    // ---- stream this warp's tiles ----------------------------------------------
    char *vt = smem + C::VT_OFF + warp * C::VTILE;             // Q8_0: dequantised V tile
    int done = 0;
    for (int i = 0; i < my_tiles; ++i) {
        const int stg = i % C::STAGES;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[stg], (i / C::STAGES) & 1, a.err, VTX_KERR_KV))) break;
        const char *st = ring + stg * C::STAGE_BYTES;
        const int n = min(KEYS, ke - (kb + (warp + W * i) * KEYS));
        if constexpr (KVT == 1) {
            decode_tile<D, C::PITCH>(st, st + KEYS * C::PITCH, n, qa, a.cx, o, m_run[0], l_part[0], lane);
        } else {
            const int qr = lane >> 2, vr = lane & 15, vh = lane >> 4;
            float sc[4];
            q8_scores<NBLK>(st + qr * C::PITCH + off, st + (qr + 8) * C::PITCH + off, qb, dq, a.cx, lane, sc);
            char *frow = vt + vr * C::FPITCH + vh * 128;
            if (vr < n) {
                dequant_2blocks(st + (KEYS + vr) * C::PITCH + off + vh * 68, frow);
            } else {
#pragma unroll
                for (int u = 0; u < 8; ++u) reinterpret_cast<uint4 *>(frow)[u] = make_uint4(0u, 0u, 0u, 0u);
            }
            __syncwarp();
            uint32_t pb[2];
            q8_softmax<D>(sc, qr < n, qr + 8 < n, o, m_run, l_part, lane, pb);
            decode_pv_t<D, C::FPITCH>(vt, pb, o, lane);
        }
        __syncwarp();                                          // every lane has read this stage
        issue(i + C::STAGES);
        done = i + 1;
    }
    // after a failed wait: this warp's copies still in flight land first (bounded)
    for (int i = done; i < min(my_tiles, done + C::STAGES); ++i)
        mbar_wait(&full[i % C::STAGES], (i / C::STAGES) & 1, nullptr, 0);

    // ---- the warps' states -> shared memory (rings are idle now) ---------------
    __syncthreads();
    float *st_o = reinterpret_cast<float *>(smem);
    float2 *st_ml = reinterpret_cast<float2 *>(smem + C::ST_ML);
    if constexpr (KVT == 1) {
        const int qrow = lane >> 2, kk = 2 * (lane & 3);
        float l = l_part[0];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        if (qrow < a.G) {
            float *so = st_o + (warp * C::GMAX + qrow) * C::SP;
            if (my_tiles > 0) {                                // an empty warp's O is never read
#pragma unroll
                for (int nb = 0; nb < NB; ++nb)
                    *reinterpret_cast<float2 *>(so + nb * 8 + kk) = make_float2(o[nb][0], o[nb][1]);
            }
            if ((lane & 3) == 0) st_ml[warp * C::GMAX + qrow] = make_float2(m_run[0], l);
        }
    } else {
        const int d0 = lane >> 2;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float l = l_part[h];
            l += __shfl_xor_sync(0xffffffffu, l, 4);
            l += __shfl_xor_sync(0xffffffffu, l, 8);
            l += __shfl_xor_sync(0xffffffffu, l, 16);
            const int hh = 2 * (lane & 3) + h;
            if (hh < a.G) {
                float *so = st_o + (warp * C::GMAX + hh) * C::SP;
                if (my_tiles > 0) {                            // an empty warp's O is never read
#pragma unroll
                    for (int j = 0; j < NJ; ++j) {
                        so[16 * j + d0] = o[j][h];
                        so[16 * j + d0 + 8] = o[j][2 + h];
                    }
                }
                if (d0 == 0) st_ml[warp * C::GMAX + hh] = make_float2(m_run[h], l);
            }
        }
    }
    __syncthreads();

    // ---- merge the warps (fixed order); final row or this split's partial ----
    // the factors 2^(m_w - M) and the row sums once per (warp, row): thread
    // r * W + w takes (row r, warp w); the row's max and sum by shuffles over
    // its W lanes (W divides 32)
    const long long work = ((long long)b * a.Hkv + g) * a.n_splits + sp;
    float *st_f = reinterpret_cast<float *>(smem + C::ST_F);
    float *cl_o = reinterpret_cast<float *>(smem + C::GRP_OFF);                        // CL: this split's
    float2 *cl_ml = reinterpret_cast<float2 *>(smem + C::GRP_OFF + C::GMAX * D * 4);   // O rows, (m, l)
    static_assert(W <= 32 && (W & (W - 1)) == 0 && C::GMAX * W % 32 == 0 && C::GMAX * W <= C::NT,
                  "a row's W lanes inside one warp, whole warps");
    if (threadIdx.x < C::GMAX * W) {
        const int r = threadIdx.x / W, w = threadIdx.x % W;
        const float2 ml = r < a.G ? st_ml[w * C::GMAX + r] : make_float2(-INFINITY, 0.f);
        float M = ml.y > 0.f ? ml.x : -INFINITY;
#pragma unroll
        for (int x = W / 2; x > 0; x >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, x));
        const float f = ml.y > 0.f ? ex2(ml.x - M) : 0.f;
        float L = f * ml.y;
#pragma unroll
        for (int x = W / 2; x > 0; x >>= 1) L += __shfl_xor_sync(0xffffffffu, L, x);
        if (r < a.G) {
            st_f[w * C::GMAX + r] = f;
            if (w == 0) {
                st_f[W * C::GMAX + r] = nsp == 1 ? (L == 0.f ? 0.f : 1.f / L) : L;
                if (nsp > 1) {
                    if constexpr (CL) cl_ml[r] = make_float2(M, L);
                    else reinterpret_cast<float2 *>(a.part_ml)[work * a.G + r] = make_float2(M, L);
                }
            }
        }
    }
    __syncthreads();
    for (int it = threadIdx.x; it < a.G * D; it += C::NT) {
        const int r = it / D, d = it % D;
        float O = 0.f;
#pragma unroll
        for (int w = 0; w < W; ++w) {
            const float f = st_f[w * C::GMAX + r];
            if (f != 0.f) O = fmaf(f, st_o[(w * C::GMAX + r) * C::SP + d], O);   // empty warps wrote no O
        }
        const float x = st_f[W * C::GMAX + r];
        if (nsp == 1) a.dst[(long long)b * a.dst_nb1 + (long long)(g * a.G + r) * D + d] = O * x;
        else if constexpr (CL) cl_o[r * D + d] = O;
        else a.part_o[(work * a.G + r) * D + d] = O;
    }
    if (nsp == 1) return;

    if constexpr (CL) {
        // ---- cluster merge: CTA sp folds the partials of all nsp splits
        //      (distributed shared memory, split order) for its share of the
        //      G x D/4 float4 outputs
        cluster_arrive();
        cluster_wait();                                        // every split's partial is in place
        const int items = a.G * (D / 4);
        const int per = (items + nsp - 1) / nsp;
        const int item = sp * per + (int)threadIdx.x;
        if ((int)threadIdx.x < per && item < items) {
            const int r = item / (D / 4), c = item % (D / 4);
            const uint32_t o_loc = smem_u32(cl_o + r * D + 4 * c);
            const uint32_t ml_loc = smem_u32(cl_ml + r);
            float2 ml[C::CLMAX];
            float4 x[C::CLMAX];
#pragma unroll
            for (int s = 0; s < C::CLMAX; ++s) {               // every load in flight at once
                ml[s] = make_float2(-INFINITY, 0.f);
                x[s] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (s < nsp) {
                    ml[s] = ld_cluster_f2(cluster_map(ml_loc, (uint32_t)s));
                    x[s] = ld_cluster_f4(cluster_map(o_loc, (uint32_t)s));
                }
            }
            float M = -INFINITY;
#pragma unroll
            for (int s = 0; s < C::CLMAX; ++s)
                if (ml[s].y > 0.f) M = fmaxf(M, ml[s].x);
            float L = 0.f;
            float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int s = 0; s < C::CLMAX; ++s) {
                if (ml[s].y > 0.f) {
                    const float f = ex2(ml[s].x - M);
                    L = fmaf(f, ml[s].y, L);
                    O.x = fmaf(f, x[s].x, O.x); O.y = fmaf(f, x[s].y, O.y);
                    O.z = fmaf(f, x[s].z, O.z); O.w = fmaf(f, x[s].w, O.w);
                }
            }
            const float inv = L == 0.f ? 0.f : 1.f / L;
            reinterpret_cast<float4 *>(a.dst + (long long)b * a.dst_nb1 + (long long)(g * a.G + r) * D)[c] =
                make_float4(O.x * inv, O.y * inv, O.z * inv, O.w * inv);
        }
        cluster_arrive();
        cluster_wait();                                        // no CTA leaves while its partial is read
        return;
    }

    // ---- split arrival; the last CTA of this (stream, KV head) merges ----------
    int *s_last = reinterpret_cast<int *>(smem + C::MISC_OFF);
    // The barrier orders every thread's partial before thread 0's arrival,
    // whose acq_rel increment at gpu scope publishes them (release is cumulative)
    // and, for the last CTA, makes every other CTA's partials visible before
    // the barrier below (the pattern of CUTLASS's split-K semaphores).
    __syncthreads();                                           // every partial of this CTA is written
    if (threadIdx.x == 0)
        *s_last = arrive_inc_acq_rel(a.flags + (long long)b * a.Hkv + g, (unsigned)(nsp - 1)) == (unsigned)(nsp - 1);
    __syncthreads();
    if (!*s_last) return;

    // thread (split group sg, item = (row, float4 column)) folds the splits
    // sg, sg + NSG, ... online; the groups are then merged in shared memory in
    // group order (the same order on every run).  Items in passes of at most
    // NT (G * D/4 may exceed the CTA's threads).
    const int items = a.G * (D / 4);
    const int per = min(items, C::NT);
    const int NSG = C::NT / per;
    const int sg = threadIdx.x / per;
    float4 *grp_o = reinterpret_cast<float4 *>(smem + C::GRP_OFF);
    float2 *grp_ml = reinterpret_cast<float2 *>(smem + C::GRP_OFF + C::NT * 16);
    const long long w0 = ((long long)b * a.Hkv + g) * a.n_splits;
    const float2 *pml = reinterpret_cast<const float2 *>(a.part_ml);
    for (int it0 = 0; it0 < items; it0 += per) {
        const int item = it0 + threadIdx.x % per;
        const int r = item / (D / 4), c = item % (D / 4);
        if (sg < NSG && item < items) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            float m_t = -INFINITY, l_t = 0.f;
            auto fold = [&](float2 ml, float4 x) {
                if (ml.y == 0.f) return;
                if (ml.x > m_t) {
                    const float f = m_t == -INFINITY ? 0.f : ex2(m_t - ml.x);
                    acc.x *= f; acc.y *= f; acc.z *= f; acc.w *= f;
                    l_t *= f;
                    m_t = ml.x;
                }
                const float w = ex2(ml.x - m_t);
                acc.x = fmaf(w, x.x, acc.x); acc.y = fmaf(w, x.y, acc.y);
                acc.z = fmaf(w, x.z, acc.z); acc.w = fmaf(w, x.w, acc.w);
                l_t = fmaf(w, ml.y, l_t);
            };
            // eight splits' loads in flight per round (predicated, not branched)
            for (int s = sg; s < nsp; s += 8 * NSG) {
                float2 mlu[8];
                float4 x[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int su = s + u * NSG;
                    mlu[u] = make_float2(-INFINITY, 0.f);
                    x[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (su < nsp) {
                        const long long wk = w0 + su;
                        mlu[u] = __ldcg(pml + wk * a.G + r);
                        x[u] = __ldcg(reinterpret_cast<const float4 *>(a.part_o + (wk * a.G + r) * D) + c);
                    }
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) fold(mlu[u], x[u]);
            }
            grp_o[threadIdx.x] = acc;
            grp_ml[threadIdx.x] = make_float2(m_t, l_t);
        }
        __syncthreads();
        if (sg == 0 && item < items) {
            const int q0 = threadIdx.x % per;
            float M = -INFINITY;
            for (int q = 0; q < NSG; ++q) {
                const float2 ml = grp_ml[q * per + q0];
                if (ml.y > 0.f) M = fmaxf(M, ml.x);
            }
            float L = 0.f;
            float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q = 0; q < NSG; ++q) {
                const float2 ml = grp_ml[q * per + q0];
                if (ml.y > 0.f) {
                    const float f = ex2(ml.x - M);
                    const float4 x = grp_o[q * per + q0];
                    L = fmaf(f, ml.y, L);
                    O.x = fmaf(f, x.x, O.x); O.y = fmaf(f, x.y, O.y);
                    O.z = fmaf(f, x.z, O.z); O.w = fmaf(f, x.w, O.w);
                }
            }
            const float inv = L == 0.f ? 0.f : 1.f / L;
            reinterpret_cast<float4 *>(a.dst + (long long)b * a.dst_nb1 + (long long)(g * a.G + r) * D)[c] =
                make_float4(O.x * inv, O.y * inv, O.z * inv, O.w * inv);
        }
        __syncthreads();                                       // the group buffers are reused by the next pass
    }
}

}  // namespace vtx
