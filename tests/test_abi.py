"""CPU tests of the C-ABI boundary: the library builds and loads, exports every
symbol include/vtx_fa.h declares, its struct layouts match the ctypes mirrors,
and operand validation answers with status codes before touching a device."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vtx_fa.h")


def declared_symbols():
    text = open(HEADER).read()
    return re.findall(r"VTX_API\s+[\w\s\*]+?\b(vtx_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    import build as b  # voxtral.cpp_b200/build.py
    b.build()
    import vtx_attn
    return vtx_attn.load()


def test_header_declares_the_entry_points():
    syms = set(declared_symbols())
    assert {"vtx_flash_attn_ext", "vtx_flash_attn_ext_workspace", "vtx_flash_attn_decode_batched",
            "vtx_flash_attn_decode_batched_workspace", "vtx_strerror", "vtx_abi_version",
            "vtx_read_device_error", "vtx_flash_attn_decode_batched_noalloc", "vtx_kv_append",
            "vtx_decode_advance", "vtx_encoder_chunk_plan", "vtx_encoder_stitch", "vtx_attn_out_proj",
            "vtx_decode_layer", "vtx_decode_layer_workspace"} <= syms


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", os.path.join(ROOT, "voxtral.cpp_b200", "libvtx_fa.so")],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    for s in declared_symbols():
        assert s in exported, s
        assert hasattr(lib, s)


def test_struct_layouts_match_ctypes(tmp_path):
    import vtx_attn
    src = tmp_path / "probe.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "vtx_fa.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(vtx_tensor),'
                   ' sizeof(vtx_fa_params), sizeof(vtx_decode_batch), offsetof(vtx_tensor, data),'
                   ' offsetof(vtx_decode_batch, q), sizeof(vtx_block_q8_0), offsetof(vtx_decode_batch, scale),'
                   ' offsetof(vtx_decode_batch, fresh_row)); return 0;}\n')
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    assert vals == [ctypes.sizeof(vtx_attn.VtxTensor), ctypes.sizeof(vtx_attn.FaParams),
                    ctypes.sizeof(vtx_attn.DecodeBatch), vtx_attn.VtxTensor.data.offset,
                    vtx_attn.DecodeBatch.q.offset, 34, vtx_attn.DecodeBatch.scale.offset,
                    vtx_attn.DecodeBatch.fresh_row.offset]


def test_kv_append_args_layout(tmp_path):
    import vtx_attn
    src = tmp_path / "probe_kv.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "vtx_fa.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu\\n", sizeof(vtx_kv_append_args),'
                   ' offsetof(vtx_kv_append_args, q), offsetof(vtx_kv_append_args, positions),'
                   ' offsetof(vtx_kv_append_args, k_cache_ptrs), offsetof(vtx_kv_append_args, cache_nb1));'
                   ' return 0;}\n')
    exe = tmp_path / "probe_kv"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    K = vtx_attn.KvAppendArgs
    assert vals == [ctypes.sizeof(K), K.q.offset, K.positions.offset, K.k_cache_ptrs.offset, K.cache_nb1.offset]


def test_kv_append_validation_without_device(lib):
    """vtx_kv_append rejects bad arguments with status codes before any device work."""
    import vtx_attn as V
    B = ctypes.byref

    def args(**kw):
        a = V.KvAppendArgs()
        a.n_tokens, a.n_head_q, a.n_head_kv, a.head_dim, a.kv_type, a.freq_base = 4, 32, 8, 128, V.F16, 1e6
        a.k, a.v, a.positions, a.slots = 0x1000, 0x2000, 0x3000, 0x4000
        a.k_nb1 = a.v_nb1 = 8 * 128 * 4
        a.k_cache, a.v_cache, a.cache_nb1 = 0x10000, 0x20000, 8 * 128 * 2
        for key, val in kw.items():
            setattr(a, key, val)
        return a

    assert lib.vtx_kv_append(None, None) == -1
    assert lib.vtx_kv_append(B(args(n_tokens=0)), None) == 0          # nothing to do, no device needed
    assert lib.vtx_kv_append(B(args(k=None)), None) == -1
    assert lib.vtx_kv_append(B(args(kv_type=30)), None) == -2
    assert lib.vtx_kv_append(B(args(head_dim=96)), None) == -5
    assert lib.vtx_kv_append(B(args(n_head_kv=0)), None) == -3
    assert lib.vtx_kv_append(B(args(k_nb1=8 * 128 * 4 + 4)), None) == -4    # rows not 8-byte aligned
    assert lib.vtx_kv_append(B(args(cache_nb1=8 * 128 * 2 + 2)), None) == -4  # F16 cache rows not 4-byte aligned
    assert lib.vtx_kv_append(B(args(q_out=0x5000)), None) == -1         # q_out without q


def test_abi_version_and_strerror(lib):
    assert lib.vtx_abi_version() == 2
    assert lib.vtx_strerror(0) == b"ok"
    assert b"workspace" in lib.vtx_strerror(-6)


def _t(lib_mod, ttype, ne, nb, ptr=0x1000):
    t = lib_mod.VtxTensor()
    t.type = ttype
    for i in range(4):
        t.ne[i], t.nb[i] = ne[i], nb[i]
    t.data = ptr
    return t


def test_validation_without_device(lib):
    """Rejected operands come back as status codes, no device involved."""
    import vtx_attn as V
    D, nq, nkv, Hq, Hkv = 64, 8, 16, 4, 2
    q = _t(V, V.F32, [D, nq, Hq, 1], [4, 4 * D * Hq, 4 * D, 4 * D * Hq * nq])
    k = _t(V, V.F16, [D, nkv, Hkv, 1], [2, 2 * D * Hkv, 2 * D, 2 * D * Hkv * nkv])
    dst = _t(V, V.F32, [D, Hq, nq, 1], [4, 4 * D, 4 * D * Hq, 4 * D * Hq * nq])
    p = V.params(0.125)
    B = ctypes.byref
    assert lib.vtx_flash_attn_ext(None, B(k), B(k), None, B(p), B(dst), None, 0, None) == -1
    bad = _t(V, 30, k.ne, k.nb)                                  # BF16: not a supported K type
    assert lib.vtx_flash_attn_ext(B(q), B(bad), B(bad), None, B(p), B(dst), None, 0, None) == -2
    k3 = _t(V, V.F16, [D, nkv, 3, 1], [2, 2 * D * 3, 2 * D, 2 * D * 3 * nkv])   # 4 % 3 != 0
    assert lib.vtx_flash_attn_ext(B(q), B(k3), B(k3), None, B(p), B(dst), None, 0, None) == -3
    q96 = _t(V, V.F32, [96, nq, Hq, 1], [4, 4 * 96 * Hq, 4 * 96, 4 * 96 * Hq * nq])
    k96 = _t(V, V.F16, [96, nkv, Hkv, 1], [2, 2 * 96 * Hkv, 2 * 96, 2 * 96 * Hkv * nkv])
    d96 = _t(V, V.F32, [96, Hq, nq, 1], [4, 4 * 96, 4 * 96 * Hq, 4 * 96 * Hq * nq])
    assert lib.vtx_flash_attn_ext(B(q96), B(k96), B(k96), None, B(p), B(d96), None, 0, None) == -5
    pw = V.params(0.125, window=10)                              # window without causal
    assert lib.vtx_flash_attn_ext(B(q), B(k), B(k), None, B(pw), B(dst), None, 0, None) == -5
    m32 = _t(V, V.F32, [nkv, nq, 1, 1], [4, 4 * nkv, 4 * nkv * nq, 4 * nkv * nq])
    assert lib.vtx_flash_attn_ext(B(q), B(k), B(k), B(m32), B(p), B(dst), None, 0, None) == -2
    assert lib.vtx_flash_attn_ext_workspace(B(q96), B(k96), B(k96), B(p)) == ctypes.c_size_t(-1).value


def test_workspace_query_is_host_only(lib):
    import vtx_attn as V
    D, nq, nkv, Hq, Hkv = 128, 1, 4096, 32, 8
    q = _t(V, V.F32, [D, nq, Hq, 1], [4, 4 * D * Hq, 4 * D, 4 * D * Hq * nq])
    k = _t(V, V.F16, [D, nkv, Hkv, 1], [2, 2 * D * Hkv, 2 * D, 2 * D * Hkv * nkv])
    n = lib.vtx_flash_attn_ext_workspace(ctypes.byref(q), ctypes.byref(k), ctypes.byref(k),
                                         ctypes.byref(V.params(0.088)))
    assert 0 < n < (1 << 30)


def test_out_proj_args_layout(tmp_path):
    import vtx_attn
    src = tmp_path / "probe_op.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "vtx_fa.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu\\n", sizeof(vtx_out_proj_args),'
                   ' offsetof(vtx_out_proj_args, block_nb), offsetof(vtx_out_proj_args, w),'
                   ' offsetof(vtx_out_proj_args, residual), offsetof(vtx_out_proj_args, dst));'
                   ' return 0;}\n')
    exe = tmp_path / "probe_op"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    A = vtx_attn.OutProjArgs
    assert vals == [ctypes.sizeof(A), A.block_nb.offset, A.w.offset, A.residual.offset, A.dst.offset]


def test_out_proj_validation_without_device(lib):
    """Shape and type errors come back before any device work."""
    import vtx_attn
    a = vtx_attn._raw_tensor(vtx_attn.F32, [64, 4, 10, 1], [4, 256, 1024, 10240], 0x1000)
    w = vtx_attn._raw_tensor(vtx_attn.F16, [256, 128, 1, 1], [2, 512], 0x1000)
    y = vtx_attn._raw_tensor(vtx_attn.F32, [128, 10, 1, 1], [4, 512], 0x1000)
    args = vtx_attn.OutProjArgs()
    args.attn, args.w, args.dst = ctypes.addressof(a), ctypes.addressof(w), ctypes.addressof(y)
    wbad = vtx_attn._raw_tensor(vtx_attn.F16, [200, 128, 1, 1], [2, 400], 0x1000)     # K != Dv * Hq
    args.w = ctypes.addressof(wbad)
    assert lib.vtx_attn_out_proj(ctypes.byref(args), None) == -3
    wf32 = vtx_attn._raw_tensor(vtx_attn.F32, [256, 128, 1, 1], [4, 1024], 0x1000)
    args.w = ctypes.addressof(wf32)
    assert lib.vtx_attn_out_proj(ctypes.byref(args), None) == -2
    assert lib.vtx_attn_out_proj(None, None) == -1


def test_decode_layer_args_layout(tmp_path):
    import vtx_attn
    src = tmp_path / "probe_dl.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "vtx_fa.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(vtx_decode_layer_args),'
                   ' offsetof(vtx_decode_layer_args, q), offsetof(vtx_decode_layer_args, positions),'
                   ' offsetof(vtx_decode_layer_args, k_cache_ptrs), offsetof(vtx_decode_layer_args, dst),'
                   ' offsetof(vtx_decode_layer_args, early)); return 0;}\n')
    exe = tmp_path / "probe_dl"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    A = vtx_attn.DecodeLayerArgs
    assert vals == [ctypes.sizeof(A), A.q.offset, A.positions.offset, A.k_cache_ptrs.offset, A.dst.offset,
                    A.early.offset]


def test_decode_layer_validation_without_device(lib):
    """Unsupported operands are rejected before any device work; the
    workspace query is host-only."""
    import vtx_attn
    a = vtx_attn.DecodeLayerArgs()
    a.n_seq, a.n_head_q, a.n_head_kv, a.head_dim, a.kv_type = 1, 32, 8, 128, vtx_attn.F32
    a.max_kv_len, a.freq_base, a.scale = 100, 1e6, 128 ** -0.5
    assert lib.vtx_decode_layer(ctypes.byref(a), None, 0, None) == -2          # F32 cache: the two-call path
    assert lib.vtx_decode_layer_workspace(ctypes.byref(a)) == ctypes.c_size_t(-1).value
    a.kv_type, a.head_dim = vtx_attn.Q8_0, 64
    assert lib.vtx_decode_layer(ctypes.byref(a), None, 0, None) == -5
    a.head_dim, a.n_head_kv, a.n_head_q = 128, 3, 12
    assert lib.vtx_decode_layer(ctypes.byref(a), None, 0, None) == -5          # Q8_0 needs an even head count
    a.n_head_kv, a.n_head_q = 2, 32
    assert lib.vtx_decode_layer(ctypes.byref(a), None, 0, None) == -5          # group of 16 > 8
    assert lib.vtx_decode_layer(None, None, 0, None) == -1
    a.n_head_kv, a.max_kv_len = 8, 7300
    n = lib.vtx_decode_layer_workspace(ctypes.byref(a))
    assert 0 < n < (1 << 24)
