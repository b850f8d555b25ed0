// Test infrastructure only: prints the reference's own encoder token counts.
//
// Built by `make -C oracle ref` from the reference's token-count functions
// (compute_causal_conv1d_dims, mel_frames_to_enc_tokens and
// compute_total_enc_tokens, src/voxtral.cpp:1274-1325, with the chunk
// constants of :26-27 and VOXTRAL_DOWNSAMPLE_FACTOR of include/voxtral.h:51),
// which the recipe extracts from the reference sources into _ref/ at build
// time; nothing of them is kept in this repository.  Reads mel frame counts
// from stdin, one per line, and prints
// "<frames> <mel_frames_to_enc_tokens> <compute_total_enc_tokens>".
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>

#include "_ref/enc_tokens_ref.inc"

int main() {
    long v;
    while (std::scanf("%ld", &v) == 1) {
        const int32_t n = (int32_t)v;
        std::printf("%d %d %d\n", n, mel_frames_to_enc_tokens(n), compute_total_enc_tokens(n));
    }
    return 0;
}
