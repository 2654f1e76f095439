"""The C ABI without a GPU: libnvllm.so loads, exports every function that
include/*.h declares, and its host-only paths (workspace sizing, status strings,
argument validation that returns before any CUDA call) behave."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
DECL = re.compile(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(nvllm_\w+)\s*\(", re.M)


HEADER_LIBS = {"nvllm.h": "libnvllm.so", "nvllm_ops.h": "libnvllm.so",
               "nvllm_host.h": "libnvllm_host.so"}


def declared(header: str) -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / header).read_text(), flags=re.S)
    return sorted(set(DECL.findall(text)))


def declared_functions() -> list[str]:
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        names += declared(h.name)
    return sorted(set(names))


def test_every_header_maps_to_a_library():
    assert sorted(h.name for h in (ROOT / "include").glob("*.h")) == sorted(HEADER_LIBS)


@pytest.mark.parametrize("header,name", [(h, n) for h in sorted(HEADER_LIBS) for n in declared(h)])
def test_library_exports_declared_symbol(header, name):
    import nvllm
    nvllm.lib()
    lib = ctypes.CDLL(str(nvllm.PKG / "lib" / HEADER_LIBS[header]))
    assert hasattr(lib, name), f"{HEADER_LIBS[header]} does not export {name}"


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("nvllm_reshape_and_cache", "nvllm_paged_attention",
                 "nvllm_paged_attention_workspace_size", "nvllm_get_last_error",
                 "nvllm_status_string"):
        assert must in names


@pytest.fixture(scope="module")
def nvlib():
    import nvllm
    return nvllm.lib()


@pytest.fixture(scope="module")
def nvmod():
    import nvllm
    nvllm.lib()
    return nvllm


def test_status_strings(nvmod):
    for code in range(7):
        assert nvmod.status_string(code) not in ("", "unknown status")
    assert nvmod.status_string(99) == "unknown status"


def test_workspace_size_host_only(nvmod):
    lay = nvmod.KVLayout(65536, 1, 16, 32, 128)
    ws = nvmod.workspace_size(64, 1, 4096, lay)
    # partials: 64 seqs x 32 heads x 16 splits x (128 floats + (m, l))
    assert ws >= 64 * 32 * 16 * (128 * 4 + 8)
    assert ws % 256 == 0
    assert nvmod.workspace_size(64, 1, 4096, nvmod.KVLayout(65536, 1, 16, 32, 48)) == 0
    assert nvmod.workspace_size(64, 1, 4096, nvmod.KVLayout(0, 1, 16, 32, 128)) == 0
    assert nvmod.workspace_size(-1, 1, 4096, lay) == 0


def test_validation_returns_before_any_launch(nvlib, nvmod):
    """Invalid geometry is refused on the host (no device pointer is touched)."""
    vp = ctypes.c_void_p
    bad_hd = nvmod.KVLayout(16, 1, 16, 2, 48)
    rc = nvlib.nvllm_reshape_and_cache(vp(16), vp(16), vp(16), vp(16), vp(16), 1, 0,
                                       ctypes.byref(bad_hd), None)
    assert rc == nvmod.ERR_UNSUPPORTED
    zero_blocks = nvmod.KVLayout(0, 1, 16, 2, 64)
    rc = nvlib.nvllm_reshape_and_cache(vp(16), vp(16), vp(16), vp(16), vp(16), 1, 0,
                                       ctypes.byref(zero_blocks), None)
    assert rc == nvmod.ERR_INVALID
    lay = nvmod.KVLayout(16, 2, 16, 2, 64)
    rc = nvlib.nvllm_reshape_and_cache(vp(16), vp(16), vp(16), vp(16), vp(16), 1, 2,
                                       ctypes.byref(lay), None)  # layer out of range
    assert rc == nvmod.ERR_INVALID
    # empty batches are no-ops that need no device
    assert nvlib.nvllm_reshape_and_cache(None, None, None, None, None, 0, 0, ctypes.byref(lay),
                                         None) == nvmod.OK
    rc = nvlib.nvllm_paged_attention(None, None, None, None, None, 1, None, None, 0, 1, 1, 0,
                                     ctypes.c_float(0.1), 0, None, 0, ctypes.byref(lay), None)
    assert rc == nvmod.OK
    # bad precision / maxima / null pointers
    args = [vp(256)] * 5
    rc = nvlib.nvllm_paged_attention(*args, 4, vp(256), vp(256), 2, 1, 64, 0,
                                     ctypes.c_float(0.1), 7, vp(256), 1 << 20,
                                     ctypes.byref(lay), None)
    assert rc == nvmod.ERR_INVALID
    rc = nvlib.nvllm_paged_attention(*args, 4, vp(256), vp(256), 2, 1, 65, 0,
                                     ctypes.c_float(0.1), 0, vp(256), 1 << 20,
                                     ctypes.byref(lay), None)  # 65 > 4 blocks x 16
    assert rc == nvmod.ERR_INVALID
    rc = nvlib.nvllm_paged_attention(None, *args[1:], 4, vp(256), vp(256), 2, 1, 64, 0,
                                     ctypes.c_float(0.1), 0, vp(256), 1 << 20,
                                     ctypes.byref(lay), None)
    assert rc == nvmod.ERR_INVALID
    rc = nvlib.nvllm_paged_attention(*args, 4, vp(256), vp(256), 2, 1, 64, 0,
                                     ctypes.c_float(0.1), 0, vp(256), 16, ctypes.byref(lay),
                                     None)  # workspace too small
    assert rc == nvmod.ERR_WORKSPACE
    rc = nvlib.nvllm_paged_attention(*args, 4, vp(256), vp(256), 2, 1, 64, 0,
                                     ctypes.c_float(0.1), 0, vp(8), 1 << 20, ctypes.byref(lay),
                                     None)  # misaligned workspace
    assert rc == nvmod.ERR_WORKSPACE


def test_model_ops_validate_on_the_host(nvlib, nvmod):
    """nvllm_ops.h entry points refuse bad arguments and treat empty work as a
    no-op without touching the device."""
    vp, i64, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
    st = None
    assert nvlib.nvllm_lcg_fill(vp(256), i64(2), i64(4), i64(3), ctypes.c_uint64(0), f32(1.0),
                                st) == nvmod.ERR_INVALID  # ld < cols
    assert nvlib.nvllm_lcg_fill(None, i64(0), i64(4), i64(4), ctypes.c_uint64(0), f32(1.0),
                                st) == nvmod.OK
    assert nvlib.nvllm_embedding_gather(vp(256), vp(256), vp(256), i64(3), i64(0), i64(8),
                                        st) == nvmod.ERR_INVALID  # empty vocabulary
    assert nvlib.nvllm_embedding_gather(None, None, None, i64(0), i64(5), i64(8), st) == nvmod.OK
    assert nvlib.nvllm_gather_rows(None, vp(256), vp(256), i64(2), i64(4), i64(8),
                                   st) == nvmod.ERR_INVALID
    assert nvlib.nvllm_rms_norm(vp(256), vp(256), None, i64(-1), i64(8), f32(1e-5),
                                st) == nvmod.ERR_INVALID
    assert nvlib.nvllm_rms_norm(None, None, None, i64(0), i64(8), f32(1e-5), st) == nvmod.OK
    assert nvlib.nvllm_silu(None, i64(4), st) == nvmod.ERR_INVALID
    assert nvlib.nvllm_add(vp(256), None, i64(4), st) == nvmod.ERR_INVALID
    assert nvlib.nvllm_penalized_argmax(vp(256), vp(256), i64(1), i64(10), f32(1.5), vp(256),
                                        None, vp(256), vp(256), ctypes.c_int32(33),
                                        st) == nvmod.ERR_INVALID  # top_k > 32
    assert nvlib.nvllm_penalized_argmax(vp(256), vp(256), i64(1), i64(10), f32(1.5), vp(256),
                                        None, None, None, ctypes.c_int32(4),
                                        st) == nvmod.ERR_INVALID  # top-k outputs missing
    # the tensor-core GEMM: shapes it does not tile are refused on the host
    outs = (ctypes.c_void_p * 1)(256)
    assert nvlib.nvllm_gemm_tf32x3(vp(256), i64(64), i64(4), i64(64), vp(256), None, i64(100), outs,
                                   ctypes.c_int32(1), i64(100), i64(100), ctypes.c_int32(0),
                                   None, ctypes.c_size_t(0), st) == nvmod.ERR_INVALID
    assert nvlib.nvllm_gemm_tf32x3(vp(256), i64(40), i64(4), i64(40), vp(256), None, i64(128), outs,
                                   ctypes.c_int32(1), i64(128), i64(128), ctypes.c_int32(3),
                                   None, ctypes.c_size_t(0), st) == nvmod.ERR_INVALID
    assert nvlib.nvllm_gemm_tf32x3(None, i64(64), i64(0), i64(64), None, None, i64(128), outs,
                                   ctypes.c_int32(1), i64(128), i64(128), ctypes.c_int32(0),
                                   None, ctypes.c_size_t(0), st) == nvmod.OK  # m = 0
    assert nvlib.nvllm_gemm_workspace_size(i64(4), i64(100), i64(64)) == 0


def test_head_gather_validates_on_the_host(nvlib, nvmod):
    """nvllm_head_gather refuses a missing group, a rank outside it, epoch 0, empty
    rows of zero width and missing peer pointers before touching the device."""
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    nvlib.nvllm_head_gather.argtypes = [vp, i64, i64, ctypes.POINTER(nvmod.HeadSplit), vp]

    def group(rank, world, epoch, fill=True):
        hs = nvmod.HeadSplit()
        hs.rank, hs.world, hs.epoch = rank, world, epoch
        for r in range(min(world, 8) if fill else 0):
            hs.outs[r] = 256 * (r + 1)
            hs.flags[r] = 4096 * (r + 1)
        return hs

    assert nvlib.nvllm_head_gather(vp(256), i64(4), i64(8), None, None) == nvmod.ERR_INVALID
    for hs in (group(2, 2, 1), group(0, 9, 1), group(0, 2, 0), group(0, 2, 1, fill=False)):
        rc = nvlib.nvllm_head_gather(vp(256), i64(4), i64(8), ctypes.byref(hs), None)
        assert rc == nvmod.ERR_INVALID
    hs = group(0, 2, 1)
    assert nvlib.nvllm_head_gather(vp(256), i64(4), i64(0), ctypes.byref(hs),
                                   None) == nvmod.ERR_INVALID  # zero width
    assert nvlib.nvllm_head_gather(None, i64(4), i64(8), ctypes.byref(hs),
                                   None) == nvmod.ERR_INVALID  # rows without data


def test_model_head_group_validates_on_the_host(nvmod):
    from nvllm.host import ModelHeadGroup, host_lib
    L = host_lib()
    L.nvllm_model_set_head_group.argtypes = [ctypes.c_void_p, ctypes.POINTER(ModelHeadGroup)]
    g = ModelHeadGroup()
    g.rank, g.world = 0, 2
    assert L.nvllm_model_set_head_group(None, ctypes.byref(g)) == nvmod.ERR_INVALID
    assert L.nvllm_model_set_head_group(ctypes.c_void_p(256), None) == nvmod.ERR_INVALID
    g.world = 9
    assert L.nvllm_model_set_head_group(ctypes.c_void_p(256), ctypes.byref(g)) == nvmod.ERR_INVALID
