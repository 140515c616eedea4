"""The reference's own Python binding, unchanged, against libcrispembed.so.

python/crispembed/_binding.py of the CrispEmbed tree is imported from the
reference checkout (skipped when the checkout is absent) and pointed at this
library through its lib_path argument:

  * CrispEmbed._setup_signatures binds every C entry point it declares without a
    hasattr() guard (python/crispembed/_binding.py:165-330): each must exist here;
  * the registry helpers it calls before a model loads (resolve_model,
    list_models, query_prefix / passage_prefix) run against this library;
  * without a GPU, CrispEmbed(path) fails the way the reference's does when
    crispembed_init returns NULL: RuntimeError("Failed to load model ...").

No device is needed; the encode path through the same binding is exercised on the
GPU by this repository's own ctypes layer (crispembed_b200/binding.py), which
declares the same argument and result types.
"""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "crispembed_b200", "libcrispembed.so")
REF_TREE = os.environ.get("CRISPEMBED_REFERENCE_TREE", "/root/reference")
REF_BINDING = os.path.join(REF_TREE, "python", "crispembed", "_binding.py")


@pytest.fixture(scope="module")
def ref_binding():
    if not os.path.exists(REF_BINDING):
        pytest.skip("reference checkout not present")
    if not os.path.exists(LIB):
        from crispembed_b200 import build
        build.build()
    spec = importlib.util.spec_from_file_location("crispembed_reference_binding", REF_BINDING)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_setup_signatures_binds_every_entry_point(ref_binding):
    obj = ref_binding.CrispEmbed.__new__(ref_binding.CrispEmbed)
    obj._lib = ref_binding._load_library(LIB)
    obj._setup_signatures()  # AttributeError if any unguarded symbol were missing
    assert obj._lib.crispembed_get_hparams.restype is not None


def test_registry_helpers(ref_binding, tmp_path):
    path = str(tmp_path / "model.gguf")
    assert ref_binding.CrispEmbed.resolve_model(path, lib_path=LIB) == path
    assert ref_binding.CrispEmbed.list_models(lib_path=LIB) == []
    assert ref_binding.CrispEmbed.query_prefix("any", lib_path=LIB) == ""
    assert ref_binding.CrispEmbed.passage_prefix("any", lib_path=LIB) == ""
    ref_binding.set_gpu_backend("cuda", lib_path=LIB)


def test_failed_init_surfaces_like_the_reference(ref_binding, tmp_path, monkeypatch):
    import torch
    if torch.cuda.is_available():
        pytest.skip("checks the no-device failure path")
    # the constructor resolves the model through the library its own search finds
    # (./build/libcrispembed.so among its paths), as a deployed copy would be found
    (tmp_path / "build").mkdir()
    os.symlink(LIB, tmp_path / "build" / "libcrispembed.so")
    monkeypatch.chdir(tmp_path)
    path = str(tmp_path / "missing.gguf")
    with pytest.raises(RuntimeError, match="Failed to load model"):
        ref_binding.CrispEmbed(path, lib_path=LIB)
