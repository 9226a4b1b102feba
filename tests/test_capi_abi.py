"""CPU checks of the C ABI: the library loads, exports exactly what include/tfattn.h declares, and
the ctypes structures match the C layout (sizes and offsets from the host C compiler)."""

import ctypes
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tfattn.h")


def _declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^TF_API [^;(]*?\b(tf_\w+)\(", src, re.M)))


def test_header_declares_every_bound_function():
    from tokenfactory_b200 import _capi
    assert _declared_functions() == sorted(n for n, _, _ in _capi.SIGNATURES)


def test_library_loads_and_exports_every_declared_symbol(tmp_path):
    from tokenfactory_b200 import _capi
    lib = _capi.load()
    for name in _declared_functions():
        assert hasattr(lib, name), name
    assert lib.tf_abi_version() == _capi.ABI_VERSION
    assert lib.tf_status_string(4).decode() == "workspace missing or too small"
    nm = shutil.which("nm")
    if nm:
        out = subprocess.run([nm, "-D", "--defined-only", _capi.LIB_PATH], capture_output=True,
                             text=True).stdout
        exported = sorted(l.split()[-1] for l in out.splitlines() if " T " in l)
        assert exported == _declared_functions(), "only the C ABI may be exported"


def test_invalid_arguments_fail_without_a_gpu():
    """Validation runs before any CUDA call: a NULL pointer is rejected with a message."""
    from tokenfactory_b200 import _capi
    lib = _capi.load()
    a = _capi.PagedAttnArgs(batch_size=2, num_tokens=2, num_q_heads=8, num_kv_heads=2,
                            head_dim=64, dtype=1)
    st = lib.tf_paged_decode_attn(ctypes.byref(a), None, 0, None)
    assert st == _capi.TF_ERR_INVALID_ARG
    assert b"NULL" in lib.tf_last_error()
    g = _capi.GdnArgs(batch_size=1, num_tokens=1)
    assert lib.tf_gdn_decode(ctypes.byref(g), None) == _capi.TF_ERR_INVALID_ARG
    p = _capi.AttnPrologueArgs(num_tokens=4, num_q_heads=8, num_kv_heads=2, head_dim=256,
                               rotary_dim=64, pos_rows=1, dtype=1)
    assert lib.tf_attn_prologue(ctypes.byref(p), None) == _capi.TF_ERR_INVALID_ARG
    assert b"NULL" in lib.tf_last_error()


_STRUCTS = {
    "tf_kv_store_args": "KVStoreArgs",
    "tf_attn_prologue_args": "AttnPrologueArgs",
    "tf_paged_attn_args": "PagedAttnArgs",
    "tf_gdn_args": "GdnArgs",
    "tf_gated_rmsnorm_args": "GatedRMSNormArgs",
    "tf_state_copy_args": "StateCopyArgs",
    "tf_r2t_sync_args": "R2TSyncArgs",
    "tf_sample_args": "SampleArgs",
    "tf_fp8_quant_args": "FP8QuantArgs",
    "tf_fp8_gemm_args": "FP8GemmArgs",
}


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs a host C compiler")
def test_ctypes_layout_matches_c(tmp_path):
    from tokenfactory_b200 import _capi
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "tfattn.h"', 'int main(void){']
    for cname, pyname in _STRUCTS.items():
        st = getattr(_capi, pyname)
        lines.append(f'printf("{pyname} size %zu\\n", sizeof({cname}));')
        for fname, _ in st._fields_:
            lines.append(f'printf("{pyname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0;}")
    c = tmp_path / "layout.c"
    c.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(c), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    for line in out.splitlines():
        pyname, field, value = line.split()
        st = getattr(_capi, pyname)
        got = ctypes.sizeof(st) if field == "size" else getattr(st, field).offset
        assert got == int(value), f"{pyname}.{field}: ctypes {got} != C {value}"


def test_prologue_rejects_unbuilt_rotary_dims_without_a_gpu():
    """Argument checks of tf_attn_prologue run before any CUDA call (fake non-NULL pointers)."""
    from tokenfactory_b200 import _capi
    lib = _capi.load()
    fake = 0x1000
    p = _capi.AttnPrologueArgs(
        q=fake, k=fake, v=fake, q_norm_weight=fake, k_norm_weight=fake, positions=fake,
        inv_freq=fake, q_out=fake, k_buffer=fake, v_buffer=fake, out_cache_loc=fake,
        num_slots=8, num_tokens=4, num_q_heads=8, num_kv_heads=2, head_dim=256, rotary_dim=48,
        pos_rows=1, dtype=1)
    assert lib.tf_attn_prologue(ctypes.byref(p), None) == _capi.TF_ERR_UNSUPPORTED
    assert b"rotary_dim 48" in lib.tf_last_error()
    p.rotary_dim, p.pos_rows = 64, 2
    assert lib.tf_attn_prologue(ctypes.byref(p), None) == _capi.TF_ERR_INVALID_ARG
    p.pos_rows = 3
    p.mrope_section[0], p.mrope_section[1], p.mrope_section[2] = 11, 11, 11
    assert lib.tf_attn_prologue(ctypes.byref(p), None) == _capi.TF_ERR_INVALID_ARG
    assert b"mrope_section" in lib.tf_last_error()


def test_state_slots_copy_checks_without_a_gpu():
    """tf_state_slots_copy validates before any CUDA call (fake non-NULL pointers): missing slot
    lists, overlapping slot rows and unknown dtypes are rejected; empty work is a no-op."""
    from tokenfactory_b200 import _capi
    lib = _capi.load()
    fake = 0x1000
    base = dict(conv_state=fake, conv_stride_layer=7 * 96, conv_stride_slot=96, conv_slot_elems=96,
                conv_dtype=1, ssm_state=fake, ssm_stride_layer=7 * 1024, ssm_stride_slot=1024,
                ssm_slot_elems=1024, ssm_dtype=0, num_layers=3, num_slots=7, num_ops=2)
    a = _capi.StateCopyArgs(**base)
    assert lib.tf_state_slots_copy(ctypes.byref(a), None) == _capi.TF_ERR_INVALID_ARG
    assert b"slot lists" in lib.tf_last_error()
    a = _capi.StateCopyArgs(**{**base, "src_slots": fake, "dst_slots": fake,
                               "ssm_stride_layer": 2048})
    assert lib.tf_state_slots_copy(ctypes.byref(a), None) == _capi.TF_ERR_INVALID_ARG
    assert b"overlap" in lib.tf_last_error()
    a = _capi.StateCopyArgs(**{**base, "src_slots": fake, "dst_slots": fake, "conv_dtype": 9})
    assert lib.tf_state_slots_copy(ctypes.byref(a), None) == _capi.TF_ERR_INVALID_ARG
    assert b"dtype" in lib.tf_last_error()
    a = _capi.StateCopyArgs(**{**base, "src_slots": fake, "dst_slots": fake, "conv_slot_elems": 97})
    assert lib.tf_state_slots_copy(ctypes.byref(a), None) == _capi.TF_ERR_INVALID_ARG
    for empty in ({"num_ops": 0}, {"num_layers": 0}, {"conv_state": None, "ssm_state": None}):
        a = _capi.StateCopyArgs(**{**base, **empty})
        assert lib.tf_state_slots_copy(ctypes.byref(a), None) == _capi.TF_OK


def test_torch_extension_loads_over_the_library_and_refuses_cpu_tensors():
    """tokenfactory_b200._C (the PyTorch front end) imports without a GPU, is linked to the same
    libtfattn.so, binds one function per ops entry point, and rejects CPU tensors before any
    launch (no CPU fallback)."""
    import torch
    from tokenfactory_b200 import _C, _capi, ops
    assert _C.ABI_VERSION == _capi.ABI_VERSION
    for name in ("kv_store", "attn_prologue", "paged_decode", "paged_extend", "gdn_decode",
                 "gdn_extend", "gated_rmsnorm", "state_slots_copy", "req_to_token_sync",
                 "sample_tokens", "fp8_quantize", "fp8_block_gemm"):
        assert callable(getattr(_C, name)), name
        assert callable(getattr(ops, name)), name
    maps = open(f"/proc/{os.getpid()}/maps").read()
    assert os.path.realpath(_capi.LIB_PATH) in maps and os.path.realpath(_C.__file__) in maps
    q = torch.zeros((2, 8, 64), dtype=torch.bfloat16)
    i = torch.zeros(2, dtype=torch.int64)
    with pytest.raises(ValueError, match="CUDA"):
        ops.paged_decode(q, q, q, i.view(1, 2), i, i, 0.125, 1)
    with pytest.raises(ValueError, match="CUDA"):
        ops.kv_store(q, q, i, q, q)
