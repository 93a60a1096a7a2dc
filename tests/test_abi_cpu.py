"""The C ABI library without a GPU: it loads, exports every declared
symbol, its struct layouts match the bindings, and calls fail loudly (no
CPU fallback) when no device is present."""
import ctypes
import os
import re

import pytest

from conftest import cuda_ok
from chonklm_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "chonk_b200.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ck_[a-z0-9_]+)\s*\(", src)))


def test_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(L, n), f"missing export {n}"


def test_struct_layouts_match():
    cfg, samp = _lib.abi_info()
    assert cfg == ctypes.sizeof(_lib.ck_model_cfg)
    assert samp == ctypes.sizeof(_lib.ck_sampling)


def test_ts_binding_layouts_match_the_abi():
    """The Bun FFI binding (chonklm_b200/ts/llama-cuda-runtime.ts) packs
    ck_model_cfg and ck_sampling by hand: its offset tables and sizes must be
    the C layout (no JavaScript runtime here to run the file itself)."""
    src = open(os.path.join(os.path.dirname(_lib.__file__), "ts", "llama-cuda-runtime.ts")).read()

    def table(name):
        body = re.search(name + r" = \{(.*?)\} as const", src, re.S).group(1)
        return {k: int(v) for k, v in re.findall(r"(\w+): (\d+)", body)}

    for cls, tname, sname in [(_lib.ck_model_cfg, "CK_CFG_LAYOUT", "CK_CFG_SIZE"),
                              (_lib.ck_sampling, "CK_SAMPLING_LAYOUT", "CK_SAMPLING_SIZE")]:
        t = table(tname)
        assert t == {f[0]: getattr(cls, f[0]).offset for f in cls._fields_}
        assert int(re.search(sname + r" = (\d+)", src).group(1)) == ctypes.sizeof(cls)
    # every symbol the binding opens is declared in the header
    opened = set(re.findall(r"^  (ck_[a-z_]+): \{", src, re.M))
    assert opened and opened <= set(declared())


def test_library_is_sm100a_and_in_tree():
    from chonklm_b200 import build
    assert os.path.dirname(_lib.lib()._name) == os.path.dirname(build.LIB)
    assert "arch=compute_100a,code=sm_100a" in " ".join(build.FLAGS)


@pytest.mark.skipif(cuda_ok(), reason="checks the no-GPU failure path")
def test_fails_loudly_without_gpu():
    c = _lib.ck_model_cfg()
    c.hidden, c.intermediate, c.vocab, c.layers = 256, 512, 1000, 2
    c.heads, c.kv_heads, c.head_dim, c.context_length = 4, 2, 64, 64
    with pytest.raises(_lib.CkError):
        _lib.Engine(c)
    with pytest.raises(_lib.CkError):
        _lib.dequant(12, bytes(144), 256, 1)


def test_config_validation_before_device():
    c = _lib.ck_model_cfg()
    c.hidden, c.intermediate, c.vocab, c.layers = 250, 512, 1000, 2     # hidden % 32 != 0
    c.heads, c.kv_heads, c.head_dim, c.context_length = 4, 2, 64, 64
    with pytest.raises(_lib.CkError, match="hidden"):
        _lib.Engine(c)
    c.hidden, c.head_dim = 256, 96
    with pytest.raises(_lib.CkError, match="head_dim"):
        _lib.Engine(c)
    c.head_dim, c.heads, c.kv_heads = 256, 8, 1                           # group 8 x 256 > 1024
    with pytest.raises(_lib.CkError, match="GQA"):
        _lib.Engine(c)


def test_product_never_imports_oracle():
    pkg = os.path.join(os.path.dirname(os.path.dirname(__file__)), "chonklm_b200")
    for root, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                txt = open(os.path.join(root, f)).read()
                assert "oracle" not in re.sub(r"#.*|//.*", "", txt).replace("Oracle", ""), f
