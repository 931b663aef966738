"""The C-ABI library: loads, exports every symbol include/llama_int4_b200.h
declares, and rejects bad arguments with status codes before any launch.
Runs without a GPU (no kernel is launched)."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "llama_int4_b200.h")


@pytest.fixture(scope="module")
def native():
    import build  # llama-efficient-inference_b200/build.py

    build.build()
    from llama import _native

    return _native


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(li4_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "li4_int4_linear" in names and "li4_quantize" in names and "li4_dequantize" in names


def test_library_exports_every_declared_symbol(native):
    lib = native.lib()
    names = declared_functions()
    for name in names:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert set(names) == set(native.SIGNATURES), "ctypes signature table out of sync with the header"


def test_version(native):
    v = native.lib().li4_version()
    assert v >> 16 == 0 and (v >> 8) & 0xFF >= 2  # 0.2: the li4_fusion layout with the argmax fields


def call_linear(native, M=1, N=64, K=256, group=128, x=16, packed=16, scale=16, zero=16, y=16,
                sxm=None, spn=None, ssn=None, sym=None, ws=None, ws_len=0):
    lib = native.lib()
    return lib.li4_int4_linear(x, packed, scale, zero, y, M, N, K, group,
                               K if sxm is None else sxm, K // 2 if spn is None else spn,
                               max(1, K // group) if ssn is None else ssn, N if sym is None else sym,
                               ws, ws_len, None)


def test_rejects_m_above_16(native):
    assert call_linear(native, M=17) == native.LI4_ERR_INVALID_ARG
    assert "M=17" in native.last_error()


def test_rejects_k_not_multiple_of_128(native):
    assert call_linear(native, K=96, group=32) == native.LI4_ERR_UNSUPPORTED


def test_rejects_bad_group(native):
    assert call_linear(native, K=384, group=96) == native.LI4_ERR_UNSUPPORTED
    assert call_linear(native, K=256, group=16) == native.LI4_ERR_UNSUPPORTED


def test_rejects_null_pointers(native):
    assert call_linear(native, x=0) == native.LI4_ERR_INVALID_ARG


def test_rejects_short_strides(native):
    assert call_linear(native, sxm=100) == native.LI4_ERR_INVALID_ARG


def test_rejects_unaligned_packed(native):
    assert call_linear(native, packed=17) == native.LI4_ERR_ALIGNMENT
    assert call_linear(native, spn=136) == native.LI4_ERR_ALIGNMENT  # row stride not a multiple of 16


def test_rejects_missing_workspace(native):
    # down_proj (N=2048, K=8192) at M=8: x over all of K would not fit the slab kernel's staging, so the
    # dispatcher splits K in four
    lib = native.lib()
    need = lib.li4_int4_linear_workspace_bytes(8, 2048, 8192, 128, 148)
    assert need >= 65536 + 4 * 8 * 2048 * 4
    assert lib.li4_int4_linear_workspace_bytes(1, 128256, 2048, 128, 148) == 0  # enough row tiles, no split
    rc = call_linear(native, M=8, N=2048, K=8192)
    # the SM count of a machine without a GPU falls back to 148, so split-K is chosen
    assert rc == native.LI4_ERR_WORKSPACE


def test_workspace_bytes_invalid_shape_is_zero(native):
    assert native.lib().li4_int4_linear_workspace_bytes(17, 64, 256, 128, 148) == 0


def test_quantize_dequantize_validate(native):
    lib = native.lib()
    assert lib.li4_quantize(16, 0, 16, 16, 16, 4, 100, 128, 100, None) == native.LI4_ERR_INVALID_ARG
    assert lib.li4_quantize(16, 9, 16, 16, 16, 4, 256, 128, 256, None) == native.LI4_ERR_INVALID_ARG
    assert lib.li4_dequantize(0, 16, 16, 16, 4, 256, 128, 128, 2, 256, None) == native.LI4_ERR_INVALID_ARG
    assert lib.li4_quantize(16, 0, 16, 16, 16, 0, 256, 128, 256, None) == native.LI4_OK  # empty: no launch


def test_fused_rejects_bad_epilogues(native):
    """li4_int4_linear_fused validates its fusion descriptor before any launch."""
    import ctypes

    lib = native.lib()

    def call(f, N=64, K=256, y=16, sym=None):
        return lib.li4_int4_linear_fused(16, 16, 16, 16, y, 1, N, K, 128, K, K // 2, K // 128,
                                         N if sym is None else sym, ctypes.byref(f), None, 0, None)

    assert call(native.Fusion(epilogue=99)) == native.LI4_ERR_INVALID_ARG
    assert call(native.Fusion(epilogue=native.LI4_EPI_RESIDUAL)) == native.LI4_ERR_INVALID_ARG  # no residual
    assert call(native.Fusion(epilogue=native.LI4_EPI_SWIGLU), N=40) == native.LI4_ERR_INVALID_ARG  # N % 16
    assert call(native.Fusion(epilogue=native.LI4_EPI_QKV_ROPE, q_rows=32, k_rows=16, head_dim=16), N=80) == \
        native.LI4_ERR_INVALID_ARG  # N != q + 2k
    assert call(native.Fusion(epilogue=native.LI4_EPI_QKV_ROPE, q_rows=32, k_rows=16, head_dim=16), N=64) == \
        native.LI4_ERR_INVALID_ARG  # no position, tables, q output or cache
    assert call(native.Fusion(norm_weight=24, epilogue=native.LI4_EPI_STORE)) == native.LI4_ERR_ALIGNMENT
    assert call(native.Fusion(epilogue=native.LI4_EPI_STORE_F32), y=18) == native.LI4_ERR_ALIGNMENT


def test_fused_allreduce_epilogue_validates(native):
    """LI4_EPI_ALLREDUCE_RESIDUAL checks its rank, buffers and sizes before any launch."""
    lib = native.lib()
    N, K, M = 64, 256, 1
    need = 2 * (N // 16) * M * 8 * 8  # world x tiles x M x 8 words of 8 bytes
    ptrs = (ctypes.c_void_p * 2)(256, 512)

    def call(N=N, world=2, rank=0, recv=ptrs, nbytes=need, epochs=1024, residual=2048):
        f = native.Fusion(epilogue=native.LI4_EPI_ALLREDUCE_RESIDUAL, residual=residual, stride_rm=N,
                          ar_recv=ctypes.cast(recv, ctypes.c_void_p), ar_recv_bytes=nbytes, ar_epochs=epochs,
                          ar_world=world, ar_rank=rank)
        return lib.li4_int4_linear_fused(16, 16, 16, 16, 16, M, N, K, 128, K, K // 2, K // 128, N,
                                         ctypes.byref(f), None, 0, None)

    assert call(world=9) == native.LI4_ERR_INVALID_ARG
    assert call(rank=2) == native.LI4_ERR_INVALID_ARG
    assert call(nbytes=need - 8) == native.LI4_ERR_INVALID_ARG
    assert call(N=40) == native.LI4_ERR_INVALID_ARG  # N % 16
    assert call(residual=0) == native.LI4_ERR_INVALID_ARG
    assert call(epochs=1026) == native.LI4_ERR_INVALID_ARG  # epoch array not 4-byte aligned
    assert call(recv=(ctypes.c_void_p * 2)(256, 516)) == native.LI4_ERR_ALIGNMENT


def test_argmax_allreduce_validates(native):
    lib = native.lib()
    rows, world = 4, 2
    need = 2 * world * rows * 2 * 8
    ptrs = (ctypes.c_void_p * 2)(256, 512)

    def call(world=world, rank=0, recv=ptrs, nbytes=need, offset=0):
        return lib.li4_argmax_rows_allreduce(256, native.LI4_F32, rows, 1000, 1000, offset,
                                             ctypes.cast(recv, ctypes.c_void_p), nbytes, 1024, world, rank, 256, 1,
                                             None)

    assert call(world=0) == native.LI4_ERR_INVALID_ARG
    assert call(rank=3) == native.LI4_ERR_INVALID_ARG
    assert call(nbytes=need - 8) == native.LI4_ERR_INVALID_ARG
    assert call(offset=-1) == native.LI4_ERR_INVALID_ARG
    assert call(recv=(ctypes.c_void_p * 2)(256, 514)) == native.LI4_ERR_ALIGNMENT


def test_grouped_validates(native):
    """li4_int4_linear_grouped_* reject bad problem lists before any copy or launch."""
    lib = native.lib()

    def probs(**kw):
        base = dict(x=256, packed=512, scale=768, zero=1024, y=1280, N=64, K=256, stride_xm=256, stride_pn=128,
                    stride_sn=2, stride_ym=64)
        base.update(kw)
        arr = (native.GemvProblem * 1)()
        arr[0] = native.GemvProblem(**base)
        return arr

    units = ctypes.c_int()
    assert lib.li4_int4_linear_grouped_table_bytes(probs(), 1, 1, ctypes.byref(units)) > 0 and units.value == 1
    assert lib.li4_int4_linear_grouped_table_bytes(probs(), 1, 9, None) == 0          # M above 8
    assert lib.li4_int4_linear_grouped_table_bytes(probs(K=200), 1, 1, None) == 0     # K % 128
    assert lib.li4_int4_linear_grouped_table_bytes(probs(K=16384 + 128, stride_xm=16512, stride_pn=8256,
                                                         stride_sn=129), 1, 1, None) == 0  # x staging
    assert lib.li4_int4_linear_grouped_build(probs(y=0), 1, 1, 128, 4096, 1 << 20) == native.LI4_ERR_INVALID_ARG
    assert lib.li4_int4_linear_grouped_build(probs(packed=520), 1, 1, 128, 4096, 1 << 20) == native.LI4_ERR_ALIGNMENT
    assert lib.li4_int4_linear_grouped_build(probs(), 1, 1, 64, 4096, 1 << 20) == native.LI4_ERR_UNSUPPORTED
    assert lib.li4_int4_linear_grouped_build(probs(), 1, 1, 128, 4096, 16) == native.LI4_ERR_WORKSPACE  # table
    assert lib.li4_int4_linear_grouped(None, 1, 1, 1, None) == native.LI4_ERR_INVALID_ARG


def grouped_ranges_mirror(shapes, wave=296):
    """The range cut of li4_int4_linear_grouped_build (li4_grouped.cu grouped_ranges), for lists whose
    x staging never forces an extra cut: each tile starts a new range when its starting kstep count
    crosses a multiple of the target (the wave's share, rounded up to a multiple of 512)."""
    tiles = [(N + 15) // 16 for N, K in shapes]
    costs = [K // 128 for N, K in shapes]
    total = sum(t * c for t, c in zip(tiles, costs))
    target = max(64, -(-total // wave))
    if target >= 512:
        target = -(-target // 512) * 512
    ranges, cost, part = [], 0, None
    for t, c in zip(tiles, costs):
        for _ in range(t):
            if part != cost // target:
                ranges.append([])
                part = cost // target
            ranges[-1].append(c)
            cost += c
    return ranges


def test_grouped_ranges_balanced(native):
    """The grouped launch's ranges for the 113 Llama-3.2-1B decode GEMVs (no GPU: a 148-SM wave of
    296 CTAs): 295 ranges, and within every range each of the 8 warps gets the same kstep count --
    the slowest warp of the slowest range sets the launch's time."""
    lib = native.lib()
    shapes = [(2048, 2048), (512, 2048), (512, 2048), (2048, 2048), (8192, 2048), (8192, 2048),
              (2048, 8192)] * 16 + [(128256, 2048)]
    arr = (native.GemvProblem * len(shapes))()
    for i, (N, K) in enumerate(shapes):
        arr[i] = native.GemvProblem(x=256, packed=512, scale=768, zero=1024, y=1280, N=N, K=K, stride_xm=K,
                                    stride_pn=K // 2, stride_sn=K // 128, stride_ym=N)
    units = ctypes.c_int()
    assert lib.li4_int4_linear_grouped_table_bytes(arr, len(shapes), 1, ctypes.byref(units)) > 0
    ranges = grouped_ranges_mirror(shapes)
    assert units.value == len(ranges) == 295
    per_warp = [max(sum(r[w::8]) for w in range(8)) for r in ranges]
    assert max(per_warp) == 256  # 2048 ksteps per range, 256 per warp
    assert sum(map(sum, ranges)) == sum(((N + 15) // 16) * (K // 128) for N, K in shapes)


def test_dispatch_plans_b200(native):
    """The automatic kernel choice on a 148-SM B200 for the Llama-3.2-1B decode shapes (from a measured
    sweep of every family and split at M = 1..16): streaming warps for the narrow shapes at every M,
    the bulk-copy ring for gate / up at M >= 2 and the fused gate-up at every M, the tile kernel for
    lm_head at M <= 8 and the bulk ring at M = 16, the shared-memory ring for down at M <= 4."""
    want = {
        (2048, 2048): ["stream"] * 5,                        # q / o
        (512, 2048): ["stream"] * 5,                         # k / v
        (3072, 2048): ["stream"] * 5,                        # fused qkv
        (2048, 8192): ["ring"] * 3 + ["stream"] * 2,         # down
        (8192, 2048): ["stream"] + ["bulk"] * 4,             # gate / up
        (16384, 2048): ["bulk"] * 5,                         # fused gate-up
        (128256, 2048): ["tile"] * 4 + ["bulk"],             # lm_head
    }
    for (N, K), kernels in want.items():
        got = [native.plan(M, N, K, 128, 148)["kernel"] for M in (1, 2, 4, 8, 16)]
        assert got == kernels, (N, K, got)


def test_attention_and_argmax_validate(native):
    lib = native.lib()
    # head_dim 48 unsupported; GQA ratio 3 unsupported; misaligned cache
    assert lib.li4_decode_attention(16, 256, 16, 16, 64 * 4 * 48, 4 * 48, 16, 256, 1, 4, 4, 48, 16, 64, None) == \
        native.LI4_ERR_UNSUPPORTED
    assert lib.li4_decode_attention(16, 384, 16, 16, 64 * 2 * 64, 2 * 64, 16, 384, 1, 6, 2, 64, 16, 64, None) == \
        native.LI4_ERR_UNSUPPORTED
    assert lib.li4_decode_attention(16, 256, 24, 16, 64 * 64, 64, 16, 256, 1, 4, 1, 64, 16, 64, None) == \
        native.LI4_ERR_ALIGNMENT
    assert lib.li4_argmax_rows(16, 7, 1, 10, 10, 16, 1, None) == native.LI4_ERR_UNSUPPORTED
    assert lib.li4_argmax_rows(16, native.LI4_F16, 1, 10, 5, 16, 1, None) == native.LI4_ERR_INVALID_ARG


def test_allreduce_validates(native):
    import ctypes

    lib = native.lib()
    arr = (ctypes.c_void_p * 9)(*([16] * 9))
    assert lib.li4_allreduce_add(arr, arr, 16, 16, 9, 0, 64, 16, 16, None) == native.LI4_ERR_INVALID_ARG  # > 8 ranks
    assert lib.li4_allreduce_add(arr, arr, 16, 16, 2, 2, 64, 16, 16, None) == native.LI4_ERR_INVALID_ARG  # rank
    odd = (ctypes.c_void_p * 2)(18, 16)
    assert lib.li4_allreduce_add(odd, arr, 16, 16, 2, 0, 64, 16, 16, None) == native.LI4_ERR_ALIGNMENT


def test_gather_rows_validates(native):
    lib = native.lib()
    assert lib.li4_gather_rows(256, 1000, 2044, 2044, 256, 1, 256, 2044, None) == native.LI4_ERR_INVALID_ARG  # cols % 8
    assert lib.li4_gather_rows(264, 1000, 2048, 2048, 256, 1, 256, 2048, None) == native.LI4_ERR_ALIGNMENT
    assert lib.li4_gather_rows(256, 1000, 2048, 2048, 256, 70000, 256, 2048, None) == native.LI4_ERR_INVALID_ARG
    assert lib.li4_gather_rows(256, 1000, 2048, 2048, 256, 0, 256, 2048, None) == native.LI4_OK  # nothing to do


def test_program_builder_validates(native):
    """Decode-program ops are checked when they are added (no GPU needed); launching an
    unfinalized program is refused."""
    import ctypes

    lib = native.lib()
    h = ctypes.c_void_p()
    assert lib.li4_program_create(ctypes.byref(h)) == native.LI4_OK
    idx = ctypes.c_int(-7)
    try:
        def lin(M=1, N=2048, K=2048, group=128, ps=1024, ss=16, scale=256, wait=-1):
            return lib.li4_program_add_linear(h, 256, 256, scale, 256, 256, M, N, K, group, K, ps, ss, N, None, wait,
                                              ctypes.byref(idx))

        assert lin() == native.LI4_OK and idx.value == 0
        assert lin(wait=0) == native.LI4_OK and idx.value == 1
        assert lin(wait=5) == native.LI4_ERR_INVALID_ARG          # waits for a later op
        assert lin(M=17) == native.LI4_ERR_UNSUPPORTED
        assert lin(N=8) == native.LI4_ERR_UNSUPPORTED             # fewer rows than a tile
        assert lin(K=3072, ps=1536, ss=24) == native.LI4_ERR_UNSUPPORTED  # K > 2048 not a multiple of 2048
        assert lin(group=64, ss=32) == native.LI4_ERR_UNSUPPORTED
        assert lin(scale=264) == native.LI4_ERR_ALIGNMENT         # scale rows off 16 bytes
        assert lin(K=512, ps=512, ss=8) == native.LI4_ERR_ALIGNMENT  # strided rows of K < 1024
        assert lin(K=8192, ps=4096, ss=64) == native.LI4_OK       # K ranges of 2048
        # attention: head_dim 48, rep 3, a context too long for the CTA's shared memory
        att = lib.li4_program_add_attention
        assert att(h, 256, 256, 256, 256, 64 * 256, 256, 256, 256, 1, 4, 1, 48, 256, 64, -1, None) == \
            native.LI4_ERR_UNSUPPORTED
        assert att(h, 256, 384, 256, 256, 64 * 128, 128, 256, 384, 1, 6, 2, 64, 256, 64, -1, None) == \
            native.LI4_ERR_UNSUPPORTED
        assert att(h, 256, 2048, 256, 256, 100000 * 512, 512, 256, 2048, 1, 32, 8, 64, 256, 100000, -1, None) == \
            native.LI4_ERR_UNSUPPORTED
        assert att(h, 256, 2048, 256, 256, 640 * 512, 512, 256, 2048, 1, 32, 8, 64, 256, 640, 1,
                   ctypes.byref(idx)) == native.LI4_OK
        assert lib.li4_program_add_gather(h, 256, 1000, 2044, 2044, 256, 1, 256, 2044, -1, None) == \
            native.LI4_ERR_INVALID_ARG                             # rows of cols % 8 != 0
        assert lib.li4_program_add_argmax(h, 256, 2, 1000, 999, 256, 1, -1, None) == native.LI4_ERR_INVALID_ARG
        assert lib.li4_program_add_increment(h, 260) == native.LI4_ERR_ALIGNMENT
        assert lib.li4_program_launch(h, None) == native.LI4_ERR_INVALID_ARG  # not finalized
    finally:
        assert lib.li4_program_destroy(h) == native.LI4_OK


def test_fusion_struct_layout_matches_header(native, tmp_path):
    """The ctypes Fusion structure has the size and field offsets of the header's li4_fusion
    (compiled with the host C compiler)."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no host C compiler")
    fields = [name for name, _ in native.Fusion._fields_]
    src = tmp_path / "layout.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "llama_int4_b200.h"\nint main(void) {\n'
                   '  printf("%zu\\n", sizeof(li4_fusion));\n' +
                   "".join(f'  printf("%zu\\n", offsetof(li4_fusion, {f}));\n' for f in fields) + "  return 0;\n}\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()]
    assert got[0] == ctypes.sizeof(native.Fusion)
    for f, off in zip(fields, got[1:]):
        assert getattr(native.Fusion, f).offset == off, f
