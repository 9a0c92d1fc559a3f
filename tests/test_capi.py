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


# ---- tensor-parallel selector, rows, attention, elementwise: host-side argument checks -----------

def _norms_call(**over):
    a = dict(k1=256, v1=256, fst=128, fsh=1024, K1=256, V1=256, cst=128, csh=4096, T=32, pos=256, n=8, H=2,
             D=128, dtype=C.TREAD_BF16, out=256, ws=256)
    a.update(over)
    return C.lib().tread_deviation_head_norms(a["k1"], a["v1"], a["fst"], a["fsh"], a["K1"], a["V1"], a["cst"],
                                              a["csh"], a["T"], a["pos"], a["n"], a["H"], a["D"], a["dtype"],
                                              a["out"], a["ws"], None)


@pytest.mark.parametrize("over,needle", [
    (dict(H=0), "Hkv"), (dict(H=33), "Hkv"), (dict(D=96), "D in"), (dict(dtype=9), "dtype"),
    (dict(k1=258), "aligned"), (dict(fsh=1025), "multiples"), (dict(T=0), "T_cache"), (dict(out=None), "null"),
])
def test_deviation_head_norms_rejects_bad_arguments(over, needle):
    assert _norms_call(**over) == 1
    assert needle in C.lib().tread_last_error().decode()


def _select_call(**over):
    a = dict(norms=256, n=8, H=2, budget=2, pos=256, dev=256, sel=256, spos=256, ws=256)
    a.update(over)
    return C.lib().tread_select_head_norms(a["norms"], a["n"], a["H"], a["budget"], a["pos"], a["dev"], a["sel"],
                                           a["spos"], a["ws"], None)


@pytest.mark.parametrize("over,needle", [
    (dict(budget=9), "budget"), (dict(budget=-1), "budget"), (dict(H=0), "Hkv"), (dict(sel=None), "sel_idx"),
    (dict(ws=260), "workspace"), (dict(norms=None), "null"),
])
def test_select_head_norms_rejects_bad_arguments(over, needle):
    assert _select_call(**over) == 1
    assert needle in C.lib().tread_last_error().decode()


def test_tp_selector_empty_is_noop():
    assert _norms_call(n=0) == 0
    assert _select_call(n=0, budget=0) == 0


def _rope_rows_call(**over):
    a = dict(qkv=256, ld=(4 + 2 * 2) * 128, pos=256, R=3, Hq=4, Hkv=2, D=128, q=256, K=256, V=256, csh=128 * 16,
             T=16, by_row=0, inv=[0.5] * 64, scale=1.0, dtype=C.TREAD_BF16)
    a.update(over)
    return C.lib().tread_rope_rows(a["qkv"], a["ld"], a["pos"], a["R"], a["Hq"], a["Hkv"], a["D"], a["q"], a["K"],
                                   a["V"], a["csh"], a["T"], a["by_row"], C.f32_array(a["inv"]), a["scale"],
                                   a["dtype"], None, None)


@pytest.mark.parametrize("over,needle", [
    (dict(R=-1), "R < 0"), (dict(Hq=3), "heads"), (dict(D=3), "head_dim"), (dict(ld=100), "ld_qkv"),
    (dict(csh=10), "cache geometry"), (dict(by_row=1, T=2), "kv_by_row"), (dict(dtype=9), "dtype"),
    (dict(K=None), "null"),
])
def test_rope_rows_rejects_bad_arguments(over, needle):
    assert _rope_rows_call(**over) == 1
    assert needle in C.lib().tread_last_error().decode()


def _attn_call(**over):
    a = dict(q=256, K=256, V=256, csh=128 * 16, T=16, pos=256, R=3, Hq=4, Hkv=2, D=128, scale=0.1, out=256,
             dtype=C.TREAD_BF16, flags=0, ws=None, ws_bytes=0)
    a.update(over)
    return C.lib().tread_attn_rows(a["q"], a["K"], a["V"], a["csh"], a["T"], a["pos"], a["R"], a["Hq"], a["Hkv"],
                                   a["D"], a["scale"], a["out"], a["dtype"], a["flags"], None, a["ws"],
                                   a["ws_bytes"], None)


@pytest.mark.parametrize("over,needle", [
    (dict(R=-1), "R < 0"), (dict(Hq=3), "heads"), (dict(Hq=34, Hkv=2), "heads"), (dict(D=96), "head_dim"),
    (dict(csh=10), "cache geometry"), (dict(dtype=9), "dtype"), (dict(flags=8), "flags"), (dict(flags=6), "flags"), (dict(out=None), "null"),
    (dict(ws=264, ws_bytes=1 << 20), "workspace"),
])
def test_attn_rows_rejects_bad_arguments(over, needle):
    assert _attn_call(**over) == 1
    assert needle in C.lib().tread_last_error().decode()


def test_rows_and_attention_empty_are_noops():
    assert _rope_rows_call(R=0) == 0
    assert _attn_call(R=0) == 0


@pytest.mark.parametrize("over,needle", [
    (dict(hidden=4), "16 bytes"), (dict(x=264), "aligned"), (dict(dtype=9), "dtype"), (dict(rows=-1), "rows"),
])
def test_rmsnorm_rejects_bad_arguments(over, needle):
    a = dict(x=256, ldx=64, w=256, y=256, ldy=64, rows=2, hidden=64, eps=1e-6, dtype=C.TREAD_BF16)
    a.update(over)
    rc = C.lib().tread_rmsnorm(a["x"], a["ldx"], a["w"], a["y"], a["ldy"], a["rows"], a["hidden"], a["eps"],
                               a["dtype"], None)
    assert rc == 1
    assert needle in C.lib().tread_last_error().decode()


@pytest.mark.parametrize("over,needle", [
    (dict(inter=4), "16 bytes"), (dict(ld=64), "16 bytes"), (dict(y=264), "aligned"), (dict(dtype=9), "dtype"),
])
def test_silu_mul_rejects_bad_arguments(over, needle):
    a = dict(gu=256, ld=128, y=256, ldy=64, rows=2, inter=64, dtype=C.TREAD_BF16)
    a.update(over)
    rc = C.lib().tread_silu_mul(a["gu"], a["ld"], a["y"], a["ldy"], a["rows"], a["inter"], a["dtype"], None)
    assert rc == 1
    assert needle in C.lib().tread_last_error().decode()


@pytest.mark.parametrize("over,needle", [
    (dict(M=129), "rows above"), (dict(K=0), "K == 0"), (dict(x=0), "null"), (dict(dtype=C.TREAD_F32), "dtype"),
    (dict(x=264), "aligned"), (dict(ldx=60), "row stride"), (dict(K=60, ldx=64, ldw=64), "multiples of 8"),
    (dict(ldw=68), "multiples of 8"), (dict(ws=512 + 64), "256-byte"),
])
def test_rows_gemm_rejects_bad_arguments(over, needle):
    a = dict(x=256, ldx=64, w=256, ldw=64, bias=None, out=256, ldo=128, M=4, N=128, K=64, acc=0,
             dtype=C.TREAD_BF16, ws=None)
    a.update(over)
    rc = C.lib().tread_rows_gemm(a["x"], a["ldx"], a["w"], a["ldw"], a["bias"], a["out"], a["ldo"], a["M"], a["N"],
                                 a["K"], a["acc"], a["dtype"], None, a["ws"], 0, None)
    assert rc == 1
    assert needle in C.lib().tread_last_error().decode()


def test_rows_gemm_empty_is_noop():
    assert C.lib().tread_rows_gemm(None, 0, None, 0, None, None, 0, 0, 16, 16, 0, C.TREAD_BF16, None, None, 0,
                                   None) == 0
    assert C.lib().tread_rows_gemm(None, 0, None, 0, None, None, 0, 4, 0, 16, 0, C.TREAD_BF16, None, None, 0,
                                   None) == 0
    assert C.lib().tread_rows_gemm_workspace_bytes() % 256 == 0
