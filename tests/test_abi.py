"""The C ABI: the library loads without a GPU and exports every declared symbol,
including everything the reference's Python binding binds unconditionally."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "crispembed_b200", "libcrispembed.so")

# python/crispembed/_binding.py:165-330 binds these without hasattr() guards
REFERENCE_BINDING_REQUIRED = [
    "crispembed_init", "crispembed_free", "crispembed_set_dim", "crispembed_get_hparams", "crispembed_encode",
    "crispembed_encode_batch", "crispembed_has_sparse", "crispembed_has_colbert", "crispembed_is_reranker",
    "crispembed_encode_sparse", "crispembed_encode_multivec", "crispembed_rerank", "crispembed_colbert_score",
    "crispembed_set_prefix", "crispembed_get_prefix", "crispembed_cache_dir", "crispembed_resolve_model",
    "crispembed_n_models", "crispembed_model_name", "crispembed_model_desc", "crispembed_model_filename",
    "crispembed_model_size", "crispembed_set_gpu_backend",
]


def declared_symbols():
    names = []
    for h in ("crispembed.h", "ceb_ops.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        names += re.findall(r"(?:CRISPEMBED_API|CEB_API)\s+[\w\s\*]+?\b(\w+)\s*\(", src)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        from crispembed_b200 import build
        build.build()
    return ctypes.CDLL(LIB)


def test_declared_symbols_exported(lib):
    names = declared_symbols()
    assert len(names) > 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_reference_binding_symbols_exported(lib):
    missing = [n for n in REFERENCE_BINDING_REQUIRED if not hasattr(lib, n)]
    assert not missing, missing


def test_pure_host_entry_points(lib):
    """Entry points that need no device work."""
    lib.crispembed_colbert_score.restype = ctypes.c_float
    lib.crispembed_colbert_score.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int,
                                             ctypes.POINTER(ctypes.c_float), ctypes.c_int, ctypes.c_int]
    q = (ctypes.c_float * 4)(1, 0, 0, 1)
    d = (ctypes.c_float * 6)(1, 0, 0, 1, 0.5, 0.5)
    assert abs(lib.crispembed_colbert_score(q, 2, d, 3, 2) - 2.0) < 1e-6
    lib.crispembed_n_models.restype = ctypes.c_int
    assert lib.crispembed_n_models() == 0
    lib.crispembed_resolve_model.restype = ctypes.c_char_p
    lib.crispembed_resolve_model.argtypes = [ctypes.c_char_p, ctypes.c_int]
    assert lib.crispembed_resolve_model(b"x.gguf", 0) == b"x.gguf"
    lib.crispembed_get_hparams.restype = ctypes.c_void_p
    assert lib.crispembed_get_hparams(None) is None


def test_hparams_struct_layout():
    from crispembed_b200.binding import _Hparams
    assert ctypes.sizeof(_Hparams) == 40  # 10 x 4 bytes, src/crispembed.h:45-56
