"""CPU-side checks of the C-ABI library: it loads, exports every symbol that
include/moe_b200.h declares, and fails loudly (no CPU fallback) when no CUDA
device is present.  No compute call is made here."""
import ctypes as C
import os
import re

import pytest

import moe_b200

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "moe_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_[a-z0-9_A-Z]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(moe_b200.LIB_PATH):
        import build
        build.build()
    return C.CDLL(moe_b200.LIB_PATH)


def test_header_and_python_mirror_agree():
    assert declared_symbols() == sorted(moe_b200.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_no_torch_in_the_boundary():
    src = open(HEADER).read()
    assert "torch" not in src.lower().replace("no torch", "")
    assert "extern \"C\"" in src


def test_context_fails_loudly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(moe_b200.MoeError):
        moe_b200.Context(0)


def test_null_context_is_rejected(lib):
    moe_b200.load_library()
    L = moe_b200._lib
    assert L.moe_ctx_destroy(None) == 1
    assert L.moe_set_async(None, 1) == 1
    assert L.moe_last_error(None) == b"null context"
    assert L.moe_kernel_launches(None) == 0


def test_ep_entry_points_without_gpu(lib):
    """Communicator ids come from NCCL on the host (no GPU involved); the
    context-taking entry points refuse a null context."""
    uid = moe_b200.ep_unique_id()
    assert len(uid) == moe_b200.EP_UNIQUE_ID_BYTES and any(uid)
    assert moe_b200.ep_unique_id() != uid
    L = moe_b200.load_library()
    assert L.moe_ep_get_unique_id(None) == 1
    buf = C.create_string_buffer(128)
    assert L.moe_ep_init(None, C.addressof(buf), 0, 1) == 1
    assert L.moe_ep_finalize(None) == 1
