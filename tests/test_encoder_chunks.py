"""The realtime encoder's chunk plan and device-side stitch (§8(f) row 3).

CPU: the oracle's restatement of the chunk geometry equals the reference's own
token-count functions (tests/golden/enc_chunks.json, generated from the
reference sources by tests/golden/make_enc_chunks.py), and the library's
vtx_encoder_chunk_plan equals the oracle's walk of run_encoder_chunked
(src/voxtral.cpp:2234-2335) for every fixture length.  GPU: vtx_encoder_stitch
is bit-exact against the oracle's host stitch, and the chunks of a realtime
encoder layer run as one batched windowed-causal attention call.
"""
import ctypes
import json
import os

import numpy as np
import pytest

import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "enc_chunks.json")


def golden_rows():
    with open(GOLDEN) as f:
        return json.load(f)["rows"]


def test_oracle_token_counts_match_reference_fixture():
    rows = golden_rows()
    assert len(rows) > 200
    for mel, toks, total in rows:
        assert O.mel_frames_to_enc_tokens(mel) == toks, mel
        assert O.compute_total_enc_tokens(mel) == total, mel


def test_oracle_plan_is_consistent():
    for mel, _, total in golden_rows():
        chunks, alloc, used = O.encoder_chunk_plan(mel)
        assert alloc == total
        assert sum(c["stride"] for c in chunks) == total
        w = 0
        for i, c in enumerate(chunks):
            assert c["write_offset"] == w and c["rope_offset"] == w - c["skip"]
            assert c["skip"] == (0 if i == 0 else 750) and c["mel_offset"] == 1500 * i
            assert 0 < c["stride"] <= c["n_tokens"] - c["skip"]
            w += c["stride"]
        assert used == total // 4 * 4
    # ten minutes of audio (100 mel frames per second): 39 chunks, 30000 tokens
    chunks, total, used = O.encoder_chunk_plan(60000)
    assert (len(chunks), total, used) == (39, 30000, 30000)


@pytest.fixture(scope="module")
def lib():
    import build as b  # voxtral.cpp_b200/build.py
    b.build()
    import vtx_attn
    return vtx_attn.load()


def test_library_plan_matches_oracle(lib):
    import vtx_attn
    mels = [m for m, _, _ in golden_rows()] + [120000, 123457, 400000]
    for mel in mels:
        chunks, total, used = vtx_attn.encoder_chunk_plan(mel)
        ochunks, ototal, oused = O.encoder_chunk_plan(mel)
        assert [c.as_dict() for c in chunks] == ochunks, mel
        assert (total, used) == (ototal, oused), mel


def test_plan_errors_and_counting(lib):
    import vtx_attn
    tot, used = ctypes.c_int32(-1), ctypes.c_int32(-1)
    assert lib.vtx_encoder_chunk_plan(-1, None, 0, ctypes.byref(tot), ctypes.byref(used)) == -3   # SHAPE
    assert lib.vtx_encoder_chunk_plan(6000, None, 4, None, None) == -1                          # NULL
    assert lib.vtx_encoder_chunk_plan(6000, None, 0, None, None) == 3                           # count only
    arr = (vtx_attn.EncChunk * 2)()                                                             # short array
    assert lib.vtx_encoder_chunk_plan(6000, arr, 2, ctypes.byref(tot), ctypes.byref(used)) == 3
    assert (arr[1].write_offset, tot.value, used.value) == (1500, 3000, 3000)
    assert lib.vtx_encoder_stitch(None, 0, 0, None, 0, 16, arr, -1, None) == -3
    assert lib.vtx_encoder_stitch(None, 0, 0, None, 0, 16, arr, 0, None) == 0                   # nothing to do


def test_enc_chunk_layout(tmp_path):
    import subprocess
    import vtx_attn
    src = tmp_path / "probe.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "vtx_fa.h"\n'
                   'int main(void){printf("%zu %zu\\n", sizeof(vtx_enc_chunk), offsetof(vtx_enc_chunk, write_offset));'
                   ' return 0;}\n')
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-I", os.path.join(os.path.dirname(HERE), "include"), str(src), "-o", str(exe)],
                   check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    assert vals == [ctypes.sizeof(vtx_attn.EncChunk), vtx_attn.EncChunk.write_offset.offset]


# ---- GPU ---------------------------------------------------------------------------

def _stitch_case(mel, dim, dtype, seed):
    import torch
    import vtx_attn
    chunks, total, _ = vtx_attn.encoder_chunk_plan(mel)
    rng = np.random.default_rng(seed)
    rows = max(c.n_tokens for c in chunks)
    if dtype == np.uint8:
        src = rng.integers(0, 256, (len(chunks), rows, dim), dtype=np.uint8)
    else:
        src = rng.standard_normal((len(chunks), rows, dim)).astype(dtype)
    want = O.encoder_stitch(src, [c.as_dict() for c in chunks], total)
    dst = torch.zeros((total, dim), dtype=torch.from_numpy(src[:1, :1]).dtype, device="cuda")
    vtx_attn.encoder_stitch(torch.from_numpy(src).cuda(), chunks, dst)
    torch.cuda.synchronize()
    return dst.cpu().numpy(), want, len(chunks)


@pytest.mark.gpu
@pytest.mark.parametrize("mel,dim,dtype", [
    (13000, 1280, np.float32),     # realtime encoder rows (enc_dim 1280 f32): 16-byte copies
    (13000, 1279, np.float32),     # 5116-byte rows: 4-byte copies
    (7001, 37, np.uint8),          # odd byte rows: byte copies
    (150000, 8, np.float32),       # 99 chunks: two launches of <= 64 chunks
])
def test_gpu_stitch_bit_exact(mel, dim, dtype):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    got, want, n = _stitch_case(mel, dim, dtype, seed=mel + dim)
    assert n >= 2
    assert np.array_equal(got, want)


@pytest.mark.gpu
def test_gpu_chunks_as_one_batched_window_call():
    """A realtime encoder layer's chunks as one vtx_flash_attn_ext call (chunks
    on the batch axis, causal + window flags): every chunk matches the oracle
    with the reference's explicit window mask, and the last, shorter chunk
    padded to the common length gives the rows of the unpadded chunk (causal
    rows never see the padding)."""
    import torch
    import vtx_attn
    from vtx_cases import assert_close, make_case, to_device
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    n, W, real_last = 300, 100, 220                # scaled from 1500 tokens, window 750
    c = make_case(77, B=3, Hq=4, Hkv=4, n_q=n, n_kv=n, D=64, kv="f16", causal=1, window=W, cache=False)
    q, k, v, _ = to_device(c)
    got = vtx_attn.flash_attn_ext(q, k, v, None, c.scale, causal=True, window=W)
    torch.cuda.synchronize()
    got = got.cpu().numpy()                         # (B, n, Hq, D)
    mask = O.window_mask(n, W)
    for b in range(3):
        ref = O.flash_attn_ext(c.q[b:b + 1], c.k[b:b + 1], c.v[b:b + 1], mask, c.scale, kv_type=O.F16)
        assert_close(got[b:b + 1], ref, f"chunk {b} vs explicit window mask")
    short = O.flash_attn_ext(c.q[2:3, :, :real_last], c.k[2:3, :, :real_last], c.v[2:3, :, :real_last],
                             O.window_mask(real_last, W), c.scale, kv_type=O.F16)
    assert_close(got[2:3, :real_last], short, "padded last chunk vs unpadded")
