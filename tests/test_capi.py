"""C-ABI library: it loads without a GPU, exports every symbol include/*.h declares, and rejects
bad arguments on the host (no CUDA call is reached in these cases)."""
import ctypes
import glob
import os
import re

import pytest

from conftest import ROOT
from tread_b200 import _capi as C


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        names |= set(re.findall(r"\b(tread_\w+)\s*\(", src))
    return sorted(names)


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "tread_rope_gather_append" in syms and "tread_last_error" in syms


def test_library_exports_every_declared_symbol():
    lib = C.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in C.SIGNATURES, f"{name} has no ctypes signature in tread_b200/_capi.py"


def test_abi_version():
    assert C.lib().tread_abi_version() >= 1


def _rope_call(**over):
    args = dict(k=[16], v=[16], n=[4], delta=[3], dst0=[0], nseg=1, out_k=16, out_v=16, L=1, H=1, D=128, T=4,
                inv=[0.5] * 64, scale=1.0, dtype=C.TREAD_BF16)
    args.update(over)
    return C.lib().tread_rope_gather_append(
        C.ptr_array(args["k"]), C.ptr_array(args["v"]), C.i32_array(args["n"]), C.i64_array(args["delta"]),
        C.i64_array(args["dst0"]), args["nseg"], args["out_k"], args["out_v"], args["L"], args["H"], args["D"],
        args["T"], C.f32_array(args["inv"]), args["scale"], args["dtype"], None)


@pytest.mark.parametrize("over,needle", [
    (dict(D=96), "head_dim"),
    (dict(D=512), "head_dim"),
    (dict(dtype=7), "dtype"),
    (dict(out_k=18), "aligned"),
    (dict(k=[24]), "aligned"),
    (dict(dst0=[1]), "outside"),
    (dict(n=[-1]), "< 0"),
    (dict(delta=[1 << 24]), "2^24"),
    (dict(nseg=-1), "nseg"),
    (dict(scale=0.0), "attn_scaling"),
])
def test_rope_gather_append_rejects_bad_arguments(over, needle):
    rc = _rope_call(**over)
    assert rc == 1
    assert needle in C.lib().tread_last_error().decode()


def test_rope_gather_append_empty_is_noop():
    assert _rope_call(nseg=0) == 0
    assert _rope_call(n=[0]) == 0


def _dev_call(**over):
    a = dict(k1=256, v1=256, fst=128, fsh=1024, K1=256, V1=256, cst=128, csh=4096, T=32, pos=256, n=8, H=4,
             D=128, budget=2, dtype=C.TREAD_BF16, dev=256, sel=256, spos=256, ws=256)
    a.update(over)
    return C.lib().tread_deviation_topk(a["k1"], a["v1"], a["fst"], a["fsh"], a["K1"], a["V1"], a["cst"], a["csh"],
                                        a["T"], a["pos"], a["n"], a["H"], a["D"], a["budget"], a["dtype"], a["dev"],
                                        a["sel"], a["spos"], a["ws"], None)


@pytest.mark.parametrize("over,needle", [
    (dict(budget=9), "budget"),
    (dict(budget=-1), "budget"),
    (dict(D=96), "D in"),
    (dict(H=0), "Hkv"),
    (dict(dtype=9), "dtype"),
    (dict(k1=258), "aligned"),
    (dict(fst=130), "multiples"),
    (dict(ws=260), "workspace"),
    (dict(T=0), "T_cache"),
    (dict(sel=None), "sel_idx"),
])
def test_deviation_topk_rejects_bad_arguments(over, needle):
    assert _dev_call(**over) == 1
    assert needle in C.lib().tread_last_error().decode()


def test_deviation_topk_empty_is_noop():
    assert _dev_call(n=0, budget=0) == 0
