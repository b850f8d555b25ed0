// fa_decode_q8.cuh — HBM-streaming decode attention over a Q8_0 KV cache
// (sm_100a).
//
// The decode node of src/voxtral.cpp:1802 with the cache quantised to Q8_0
// (ggml blocks {f16 d; int8 qs[32]}, 34 bytes per 32 values): one decode token
// per stream reads every cache byte once, so the kernel is bound by HBM.
// A head's row is 136 bytes (D = 128) and only 8-byte aligned, so per-head
// rows cannot be bulk-copied.  Instead one CTA covers HPC consecutive KV heads
// (all 8 of voxtral's decoder) of one (stream, key split):
//
//   producer warp   lane l bulk-copies the HPC-head slice of token row l (K,
//                   l < 16) or l - 16 (V) of a 16-key stage into a 4-stage
//                   ring — HPC * 136 bytes, contiguous and 16-byte aligned,
//                   rows padded by 16 B; completion counted by one mbarrier
//                   per stage, reuse gated by a second one (one arrival per
//                   head warp that reads the stage).
//   head warps      two per KV head, taking alternate stages; each keeps its
//                   own softmax state and the pair merges them at the end.
//
// Per 16-key stage a head warp computes the transposed scores
// S^T (16 keys x 8 heads) with one integer MMA per 32-value block
// (mma m16n8k32 s8: A = the int8 K values, loaded straight from the ring;
// B = Q quantised to Q8_0), then s += (d_k * d_q) * isum block by block —
// ggml_vec_dot_q8_0_q8_0's arithmetic, with Q quantised first as ggml's CPU
// kernel does (d = amax/127, q = round-half-even(x * 127/amax)).  V is
// dequantised into a private f16 tile (int8 -> f16 exactly through the 0x64xx
// bit pattern, times the block scale, rounded once) and
// O^T (D x 8 heads) += V^T P^T runs with V^T as the M operand (ldmatrix.trans)
// and P^T taken from the score fragment with movmatrix.trans.  Partials use
// fa_combine_kernel's layout.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "vtx_ptx.cuh"
#include "fa_splitkv.cuh"
#include "fa_decode_mma.cuh"

namespace vtx {

template <int D> struct DecodeQ8Cfg {
    static_assert(D == 128, "Q8_0 streaming decode is built for head_dim 128");
    static constexpr int KEYS = 16;                          // keys per stage
    static constexpr int STAGES = 4;                         // ~140 KB of a CTA's rows in flight
    static constexpr int HPC_MAX = 8;                        // KV heads per CTA
    static constexpr int WPH = 2;                            // head warps per KV head (alternate stages)
    static_assert(WPH == 1 || WPH == 2, "stages alternate between at most two warps per head");
    static constexpr int NBLK = D / 32;                      // Q8_0 blocks per head row
    static constexpr int BLK = NBLK * 34;                    // one head's Q8_0 row (136 B)
    static constexpr int RPC = 4;                            // token rows per bulk copy
    static_assert(RPC == 2 || RPC == 4, "ring rows per copy");
    // MMA row m of a stage (S^T row, V tile row) -> its key within the stage.
    // Rows of one copy sit trow bytes apart (trow / 4 = 16 mod 32 banks for 8
    // heads), so rows r and r + 2 of a copy share banks; with 4 rows per copy
    // rows 0-7 take keys {4p, 4p + 1} and rows 8-15 keys {4p + 2, 4p + 3}, so
    // the eight rows one fragment load touches fall in eight bank groups.
    static __device__ __forceinline__ int key_of(int m) {
        if constexpr (RPC == 4) return 4 * ((m & 7) >> 1) + (m & 1) + 2 * (m >> 3);
        else return m;
    }
    static constexpr int RING_STAGE = 2 * KEYS / RPC * (RPC * HPC_MAX * BLK + 16);   // copies padded by 16 B
    static constexpr int FPITCH = D * 2 + 16;                // dequantised f16 row pitch
    static constexpr int MERGE = 32 * (D / 4 + 4) * 4;       // one warp's softmax state for the pair merge
    static constexpr int WBUF = KEYS * FPITCH > MERGE ? KEYS * FPITCH : MERGE;   // V tile, then merge state
    static constexpr int BUF_OFF = STAGES * RING_STAGE;
    static constexpr int BAR_OFF = BUF_OFF + HPC_MAX * WPH * WBUF;
    static constexpr int SMEM = BAR_OFF + 2 * STAGES * 8;
    static constexpr int NTHREADS = (HPC_MAX * WPH + 1) * 32;
};

// 4 int8 (one 32-bit word) -> two f16x2, each value d * q rounded to half.
__device__ __forceinline__ void q8x4_to_h2(uint32_t w, __half2 d2, uint32_t &lo, uint32_t &hi) {
    const uint32_t u = w ^ 0x80808080u;                      // q + 128, as unsigned bytes
    uint32_t a, b;
    asm("prmt.b32 %0, %1, %2, 0x5140;" : "=r"(a) : "r"(u), "r"(0x64646464u));   // {0x64, u0}, {0x64, u1}
    asm("prmt.b32 %0, %1, %2, 0x5342;" : "=r"(b) : "r"(u), "r"(0x64646464u));   // {0x64, u2}, {0x64, u3}
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));   // 1152
    __half2 fa = __hsub2(*reinterpret_cast<__half2 *>(&a), bias);    // exact q
    __half2 fb = __hsub2(*reinterpret_cast<__half2 *>(&b), bias);
    fa = __hmul2(fa, d2);                                    // exact product, one rounding
    fb = __hmul2(fb, d2);
    lo = *reinterpret_cast<uint32_t *>(&fa);
    hi = *reinterpret_cast<uint32_t *>(&fb);
}

// Half of one head's Q8_0 row: two blocks (68 bytes from a 4-byte aligned
// shared-memory address) -> 64 halves written to dst (16-byte aligned).
// The first block's int8 values sit at a 2-byte offset (funnel shifts), the
// second block's on word boundaries.
__device__ __forceinline__ void dequant_2blocks(const char *src, char *dst) {
    uint32_t w[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) w[i] = reinterpret_cast<const uint32_t *>(src)[i];
    const __half dA = __ushort_as_half((unsigned short)(w[0] & 0xffffu));   // bytes 0-1
    const __half dB = __ushort_as_half((unsigned short)(w[8] >> 16));       // bytes 34-35
    const __half2 dA2 = __halves2half2(dA, dA), dB2 = __halves2half2(dB, dB);
    uint32_t out[32];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        q8x4_to_h2(__funnelshift_r(w[j], w[j + 1], 16), dA2, out[2 * j], out[2 * j + 1]);   // bytes 2..33
        q8x4_to_h2(w[9 + j], dB2, out[16 + 2 * j], out[16 + 2 * j + 1]);                  // bytes 36..67
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
        reinterpret_cast<uint4 *>(dst)[i] = make_uint4(out[4 * i], out[4 * i + 1], out[4 * i + 2], out[4 * i + 3]);
}

// ---- one 16-key stage with the keys (S^T) and dims (O^T) as the MMA rows -----
// A lane (r = l/4, c = l%4) holds S^T for keys r and r + 8 and heads 2c, 2c+1,
// and O^T for dims 16j + r and 16j + r + 8 and the same two heads.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
// D = A (16x32 s8, row) * B (32x8 s8, col), s32, zero accumulator
__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ uint32_t lds32(const char *p) { return *reinterpret_cast<const uint32_t *>(p); }
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Four int8 of a Q8_0 block starting at byte o of a 4-byte aligned head row:
// the qs of even blocks sit 2 bytes off a word boundary (o % 4 == 2).
template <int J>
__device__ __forceinline__ uint32_t q8_word(const char *row, int o) {
    if (J & 1) return lds32(row + o);
    return __funnelshift_r(lds32(row + o - 2), lds32(row + o + 2), 16);
}

// S^T for one stage, in the log2 domain (times cx).  krow, krow8: the ring
// rows (head slices) of the keys in MMA rows r and r + 8.  qb: the s8
// B fragments of Q (head r, values 32j + 4c.. and 32j + 16 + 4c..); dq: the Q
// block scales of heads 2c, 2c+1.
template <int NBLK>
__device__ __forceinline__ void q8_scores(const char *krow, const char *krow8, const uint32_t (&qb)[NBLK][2],
                                          const float (&dq)[NBLK][2], float cx, int lane, float (&s)[4])
{
    const int c4 = 4 * (lane & 3);
    s[0] = s[1] = s[2] = s[3] = 0.f;
#pragma unroll
    for (int j = 0; j < NBLK; ++j) {
        const int o = j * 34 + 2 + c4;
        uint32_t a0, a1, a2, a3;
        if (j & 1) {
            a0 = q8_word<1>(krow, o); a1 = q8_word<1>(krow8, o);
            a2 = q8_word<1>(krow, o + 16); a3 = q8_word<1>(krow8, o + 16);
        } else {
            a0 = q8_word<0>(krow, o); a1 = q8_word<0>(krow8, o);
            a2 = q8_word<0>(krow, o + 16); a3 = q8_word<0>(krow8, o + 16);
        }
        int acc[4];
        mma_s8(acc, a0, a1, a2, a3, qb[j][0], qb[j][1]);
        const float dk0 = __half2float(*reinterpret_cast<const __half *>(krow + j * 34));
        const float dk1 = __half2float(*reinterpret_cast<const __half *>(krow8 + j * 34));
        s[0] = fmaf(dk0 * dq[j][0], (float)acc[0], s[0]);
        s[1] = fmaf(dk0 * dq[j][1], (float)acc[1], s[1]);
        s[2] = fmaf(dk1 * dq[j][0], (float)acc[2], s[2]);
        s[3] = fmaf(dk1 * dq[j][1], (float)acc[3], s[3]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) s[i] *= cx;
}

// Online softmax over the stage's keys (MMA rows whose key is past the stage
// masked: ok0 for row r, ok1 for row r + 8), per head column.
// The running max moves only when some key exceeds it by more than 2^8 (a
// warp vote; the cross-lane max is reduced only then), so P <= 256.  Returns
// P^T as the B fragment of the PV product.
template <int D>
__device__ __forceinline__ void q8_softmax(float (&s)[4], bool ok0, bool ok1, float (&o)[D / 16][4], float (&m_run)[2],
                                           float (&l_part)[2], int lane, uint32_t (&pb)[2])
{
    if (!ok0) s[0] = s[1] = -INFINITY;
    if (!ok1) s[2] = s[3] = -INFINITY;
    float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
    if (__any_sync(0xffffffffu, mx0 > m_run[0] + 8.0f || mx1 > m_run[1] + 8.0f)) {
#pragma unroll
        for (int x = 4; x < 32; x <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, x));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, x));
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float mx = h ? mx1 : mx0;
            if (mx > m_run[h] + 8.0f) {              // uniform over the lanes of this head column
                const float alpha = m_run[h] == -INFINITY ? 0.f : ex2(m_run[h] - mx);
                m_run[h] = mx;
                l_part[h] *= alpha;
#pragma unroll
                for (int j = 0; j < D / 16; ++j) {
                    o[j][h] *= alpha;
                    o[j][2 + h] *= alpha;
                }
            }
        }
    }
    float p[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const float mu = m_run[h] == -INFINITY ? 0.f : m_run[h];
        p[h] = ex2(s[h] - mu);
        p[2 + h] = ex2(s[2 + h] - mu);
        l_part[h] += p[h] + p[2 + h];
    }
    // the two 8x8 blocks (keys 0-7, keys 8-15) x heads, transposed in registers
    pb[0] = movmatrix_t(pack_half2(p[0], p[1]));
    pb[1] = movmatrix_t(pack_half2(p[2], p[3]));
}

template <int D, int PITCH>
__device__ __forceinline__ void decode_pv_t(const char *vs, const uint32_t (&pb)[2], float (&o)[D / 16][4], int lane)
{
    // ldmatrix.trans x4: lanes 0-7 keys 0-7 dims [16j, +8), 8-15 keys 0-7 dims +8,
    // 16-23 keys 8-15 dims [16j, +8), 24-31 keys 8-15 dims +8
    const char *vrow = vs + ((lane & 7) + (lane >> 4) * 8) * PITCH + ((lane >> 3) & 1) * 16;
#pragma unroll
    for (int j = 0; j < D / 16; ++j) {
        uint32_t a[4];
        ldsm_x4_t(a, vrow + j * 32);
        mma16816(o[j], a, pb[0], pb[1]);
    }
}

// Stores one lane's share: heads h0, h0 + 1 (those < G), dims l/4 (+8) of
// every 16-dim block; final normalised rows or the split's partial.
template <int D>
__device__ __forceinline__ void decode_store_t(const SplitArgs &a, int b, int g, int sp, const float (&o)[D / 16][4],
                                               const float (&m_run)[2], const float (&l_part)[2], int lane)
{
    const long long work = ((long long)b * a.Hkv + g) * a.n_splits + sp;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        float l = l_part[h];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        const int hh = 2 * (lane & 3) + h;          // head within the group
        if (hh >= a.G) continue;
        const int d0 = lane >> 2;
        if (a.write_final) {
            float *out = reinterpret_cast<float *>(a.dst + (long long)(g * a.G + hh) * a.d_nb1 +
                                                   (long long)b * a.d_nb3);
            const float inv = l == 0.f ? 0.f : 1.f / l;
#pragma unroll
            for (int j = 0; j < D / 16; ++j) {
                out[16 * j + d0] = o[j][h] * inv;
                out[16 * j + d0 + 8] = o[j][2 + h] * inv;
            }
        } else {
            float *po = a.part_o + (work * 4 + hh) * D;
#pragma unroll
            for (int j = 0; j < D / 16; ++j) {
                po[16 * j + d0] = o[j][h];
                po[16 * j + d0 + 8] = o[j][2 + h];
            }
            if (d0 == 0) {
                a.part_ml[(work * 4 + hh) * 2 + 0] = m_run[h];
                a.part_ml[(work * 4 + hh) * 2 + 1] = l;
            }
        }
    }
}

template <int D>
__global__ void __launch_bounds__(DecodeQ8Cfg<D>::NTHREADS, 1)
fa_decode_q8_kernel(const SplitArgs a, int hpc)
{
    // With a.fresh only q and one row per stream come from the kernel launched
    // just before: the producer fills the ring before waiting for it, except
    // for the stage holding that row; the head warps wait before reading q.
    const bool early = a.fresh != nullptr;
    if (!early) grid_dep_wait();
    grid_dep_launch();
    using C = DecodeQ8Cfg<D>;
    constexpr int NBLK = C::NBLK, NJ = D / 16;
    extern __shared__ __align__(128) char smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *empty = full + C::STAGES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // work item: (stream b, head group hg, key split sp)
    const int ngroups = a.Hkv / hpc;
    const int hg = blockIdx.x % ngroups;
    const int sp = (blockIdx.x / ngroups) % a.n_splits;
    const int b = blockIdx.x / (ngroups * a.n_splits);
    const int trow = hpc * C::BLK;                           // bytes of a token row's group slice
    const int cpitch = C::RPC * trow + 16;                   // ring pitch of RPC rows: copies rotate banks
    const int half_off = C::KEYS / C::RPC * cpitch;          // V rows of a stage
    // key r of a stage's K (or V) half sits at (r / RPC) * cpitch + (r % RPC) * trow
    auto ring_row = [&](int r) { return (r / C::RPC) * cpitch + (r % C::RPC) * trow; };

    int kv_len = a.n_kv;
    const char *kbase, *vbase;
    if (a.k_ptrs) {
        kv_len = a.kv_len[b];
        kbase = static_cast<const char *>(a.k_ptrs[b]);
        vbase = static_cast<const char *>(a.v_ptrs[b]);
    } else {
        kbase = a.k + (long long)(b / a.k_bdiv) * a.k_nb3;
        vbase = a.v + (long long)(b / a.v_bdiv) * a.v_nb3;
    }
    kbase += (long long)hg * hpc * a.k_nb2;
    vbase += (long long)hg * hpc * a.v_nb2;
    const int kb = sp * a.chunk;
    const int ke = min(kb + a.chunk, kv_len);
    // splits past this stream's length are not read by the combine kernel
    if (a.k_ptrs && sp > 0 && kb >= kv_len) return;
    const bool misaligned = ((reinterpret_cast<uintptr_t>(kbase) | reinterpret_cast<uintptr_t>(vbase) |
                              (uintptr_t)a.k_nb1 | (uintptr_t)a.v_nb1) & 15) != 0;
    if (misaligned && threadIdx.x == 0 && a.err) atomicCAS(a.err, 0, 7);
    const int ntiles = (ke > kb && !misaligned) ? (ke - kb + C::KEYS - 1) / C::KEYS : 0;
    // the group is the whole token row: RPC consecutive rows are one contiguous copy
    const bool contig = a.k_nb1 == trow && a.v_nb1 == trow;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], hpc);
        }
        fence_mbar_init();
    }
    __syncthreads();

    constexpr int HEAD_WARPS = C::HPC_MAX * C::WPH;
    if (warp == HEAD_WARPS) {
        // ================= producer =========================================
        const int fresh = early && a.k_ptrs ? a.fresh[b] : -1;   // row the preceding kernel writes
        bool waited = !early;
        int issued = 0;
        for (int t = 0; t < ntiles; ++t) {
            const int stg = t % C::STAGES;
            if (t >= C::STAGES &&
                !__all_sync(0xffffffffu, mbar_wait(&empty[stg], ((t / C::STAGES) - 1) & 1, a.err, VTX_KERR_KV)))
                break;
            const int k0 = kb + t * C::KEYS;
            const int n = min(C::KEYS, ke - k0);
            if (!waited && fresh >= k0 && fresh < k0 + n) {   // this stage holds the fresh row
                grid_dep_wait();
                waited = true;
            }
            char *st = smem + stg * C::RING_STAGE;
            if (lane == 0) mbar_arrive_expect_tx(&full[stg], (uint32_t)(2 * n * trow));
            __syncwarp();
            const bool isv = lane >= 16;
            const char *src = isv ? vbase : kbase;
            const long long nb1 = isv ? a.v_nb1 : a.k_nb1;
            char *dst = st + (isv ? half_off : 0);
            if (contig) {                                    // lane c < KEYS / RPC: rows RPC c ..
                const int c = lane & 15, r = c * C::RPC;
                if (c < C::KEYS / C::RPC && r < n)
                    bulk_g2s(dst + c * cpitch, src + (long long)(k0 + r) * nb1, (uint32_t)(min(C::RPC, n - r) * trow),
                             &full[stg]);
            } else {                                         // one copy per row
                const int r = lane & 15;
                if (r < n)
                    bulk_g2s(dst + (r / C::RPC) * cpitch + (r % C::RPC) * trow, src + (long long)(k0 + r) * nb1,
                             (uint32_t)trow, &full[stg]);
            }
            issued = t + 1;
        }
        // the CTA's shared memory must outlive every copy still in flight (bounded)
        for (int t = issued > C::STAGES ? issued - C::STAGES : 0; t < issued; ++t)
            mbar_wait(&full[t % C::STAGES], (t / C::STAGES) & 1, nullptr, 0);
        return;
    }
    const int hw = warp % C::HPC_MAX, par = warp / C::HPC_MAX;   // head in the group, stage parity
    if (hw >= hpc) return;

    // ==================== head warp ============================================
    const int g = hg * hpc + hw;                             // KV head
    char *buf = smem + C::BUF_OFF + warp * C::WBUF;          // dequantised V of a stage

    // Q of the group quantised to Q8_0 per 32 values (ggml's from_float for a
    // Q8_0 K): lane (r, c) holds head r's int8 values 32j + 4c.. and
    // 32j + 16 + 4c.. as the s8 B fragment; heads >= G are zero.
    const int qr = lane >> 2, qc = lane & 3;
    uint32_t qb[NBLK][2];
    float dq[NBLK][2];
    if (early) grid_dep_wait();                              // q is written by the preceding kernel
    {
        const bool rq = qr < a.G;
        const char *qp = a.q + (long long)(g * a.G + (rq ? qr : 0)) * a.q_nb2 + (long long)b * a.q_nb3;
#pragma unroll
        for (int j = 0; j < NBLK; ++j) {
            float x[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int c = 32 * j + 4 * qc + (i & 3) + (i >> 2) * 16;
                x[i] = 0.f;
                if (rq) x[i] = a.q_f16 ? __half2float(reinterpret_cast<const __half *>(qp)[c])
                                       : reinterpret_cast<const float *>(qp)[c];
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
            for (int i = 0; i < 8; ++i)
                w[i >> 2] |= ((uint32_t)__float2int_rn(x[i] * id) & 0xffu) << (8 * (i & 3));
            qb[j][0] = w[0];
            qb[j][1] = w[1];
            dq[j][0] = __shfl_sync(0xffffffffu, d, 8 * qc);          // head 2c
            dq[j][1] = __shfl_sync(0xffffffffu, d, 8 * qc + 4);      // head 2c + 1
        }
    }

    float o[NJ][4];
#pragma unroll
    for (int j = 0; j < NJ; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_part[2] = {0.f, 0.f};
    const float cx = a.qk_scale * kLog2e;
    const int vr = lane & 15, vh = lane >> 4;                // V dequant: tile row, which 2 of its 4 blocks
    char *frow = buf + vr * C::FPITCH + vh * 128;
    const int key0 = C::key_of(qr), key1 = C::key_of(qr + 8), vkey = C::key_of(vr);
    const int koff0 = ring_row(key0), koff1 = ring_row(key1), voff = half_off + ring_row(vkey) + vh * 68;

    for (int t = par; t < ntiles; t += C::WPH) {
        const int stg = t % C::STAGES;
        if (!__all_sync(0xffffffffu, mbar_wait(&full[stg], (t / C::STAGES) & 1, a.err, VTX_KERR_KV))) break;
        const int k0 = kb + t * C::KEYS;
        const int n = min(C::KEYS, ke - k0);
        const char *st = smem + stg * C::RING_STAGE + hw * C::BLK;
        // rows >= n of the stage were not loaded: their scores are masked, and
        // their V rows are zeros in the tile, so P = 0 multiplies zeros
        float sc[4];
        q8_scores<NBLK>(st + koff0, st + koff1, qb, dq, cx, lane, sc);
        if (vkey < n) {
            dequant_2blocks(st + voff, frow);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) reinterpret_cast<uint4 *>(frow)[i] = make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stg]);             // this warp is done with the ring stage
        uint32_t pb[2];
        q8_softmax<D>(sc, key0 < n, key1 < n, o, m_run, l_part, lane, pb);
        decode_pv_t<D, C::FPITCH>(buf, pb, o, lane);
        __syncwarp();                                        // V tile read before the next stage's
    }

    // merge the pair's states: the odd-stage warp hands (m, l, O) to the other
    // (the named barrier counts exactly the pair's two warps)
    if constexpr (C::WPH == 2) {
        float *ms = reinterpret_cast<float *>(smem + C::BUF_OFF + (C::HPC_MAX + hw) * C::WBUF) + lane * (D / 4 + 4);
        if (par == 1) {
#pragma unroll
            for (int j = 0; j < NJ; ++j)
                *reinterpret_cast<float4 *>(ms + 4 * j) = make_float4(o[j][0], o[j][1], o[j][2], o[j][3]);
            *reinterpret_cast<float4 *>(ms + D / 4) = make_float4(m_run[0], m_run[1], l_part[0], l_part[1]);
        }
        named_bar_sync(1 + hw, 64);
        if (par == 1) return;
        const float4 ml = *reinterpret_cast<const float4 *>(ms + D / 4);
        const float m1[2] = {ml.x, ml.y}, l1[2] = {ml.z, ml.w};
        float a0[2], a1[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float m = fmaxf(m_run[h], m1[h]);
            a0[h] = m_run[h] == -INFINITY ? 0.f : ex2(m_run[h] - m);
            a1[h] = m1[h] == -INFINITY ? 0.f : ex2(m1[h] - m);
            m_run[h] = m;
            l_part[h] = l_part[h] * a0[h] + l1[h] * a1[h];
        }
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const float4 v = *reinterpret_cast<const float4 *>(ms + 4 * j);
            o[j][0] = o[j][0] * a0[0] + v.x * a1[0];
            o[j][1] = o[j][1] * a0[1] + v.y * a1[1];
            o[j][2] = o[j][2] * a0[0] + v.z * a1[0];
            o[j][3] = o[j][3] * a0[1] + v.w * a1[1];
        }
    }
    decode_store_t<D>(a, b, g, sp, o, m_run, l_part, lane);
}

}  // namespace vtx
