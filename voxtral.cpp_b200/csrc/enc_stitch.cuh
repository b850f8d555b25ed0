// enc_stitch.cuh — device-side stitch of the realtime encoder's chunk outputs.
//
// run_encoder_chunked (src/voxtral.cpp:2234-2335) encodes overlapping chunks
// and copies each chunk's new rows [skip, skip + stride) into the long-form
// encoder output through host memory (:2318-2328).  This kernel does all the
// chunks' copies in one launch on the device: a CTA per output row at a time
// (grid-stride over the rows of up to 64 chunks), the row copied with the
// widest vector that the pointers, pitches and row size allow.  It moves
// 2 x rows x row_bytes through HBM and does nothing else.
#pragma once
#include <cstdint>
#include <type_traits>
#include "vtx_ptx.cuh"

namespace vtx {

constexpr int kStitchMaxChunks = 64;                 // chunks per launch (kernel parameter space)

struct StitchArgs {
    const char *src; long long src_chunk, src_row;   // chunk c row r at src + c*src_chunk + r*src_row
    char *dst; long long dst_row;
    long long row_bytes;
    int n;                                           // chunks in this launch
    int first[kStitchMaxChunks + 1];                 // first output row of each chunk (launch-relative), total
    int skip[kStitchMaxChunks], write[kStitchMaxChunks], chunk[kStitchMaxChunks];
};

template <int VEC>
__global__ void __launch_bounds__(256) enc_stitch_kernel(const StitchArgs a)
{
    grid_dep_wait();
    grid_dep_launch();
    using V = typename std::conditional<VEC == 16, uint4,
              typename std::conditional<VEC == 8, uint2,
              typename std::conditional<VEC == 4, uint32_t, uint8_t>::type>::type>::type;
    const int total = a.first[a.n];
    const long long nv = a.row_bytes / VEC;
    for (int row = blockIdx.x; row < total; row += gridDim.x) {
        int c = 0;
        while (c + 1 < a.n && a.first[c + 1] <= row) ++c;           // <= 64 steps, uniform over the CTA
        const int r = row - a.first[c];
        const V *s = reinterpret_cast<const V *>(a.src + (long long)a.chunk[c] * a.src_chunk +
                                                 (long long)(a.skip[c] + r) * a.src_row);
        V *d = reinterpret_cast<V *>(a.dst + (long long)(a.write[c] + r) * a.dst_row);
        for (long long i = threadIdx.x; i < nv; i += blockDim.x) d[i] = s[i];
    }
}

}  // namespace vtx
