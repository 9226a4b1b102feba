"""Block-FP8 linear (qwen3_8/fp8_triton.py) on CPU: the oracle against fixtures recorded from the
reference's own triton_block_fp8_linear (its kernel run in Triton's interpreter), the e4m3
encoder against torch's conversion (the reference's dependency), the drop-in over the
reference's functions, and the C ABI's argument checks (no GPU needed)."""

import ctypes
import inspect

import numpy as np
import pytest
import torch

from oracle import bf16 as BF
from oracle import fp8 as OF
from tests.golden import cases as C
from tests.golden.load import fp8_case


@pytest.mark.parametrize("name", sorted(C.FP8_CASES))
def test_oracle_matches_reference_fixture(name):
    spec, inp, gold = fp8_case(name)
    q, s = OF.quantize_act(inp["x"], spec["dtype"])
    np.testing.assert_array_equal(q, gold["q"])           # bit-exact activation quantization
    assert np.float32(s) == gold["x_scale"][0]
    bias = BF.as_f32(inp["bias"], spec["dtype"]) if "bias" in inp else None
    ref = OF.block_fp8_linear(gold["q"], gold["x_scale"][0], inp["w"], inp.get("w_scale"), bias)
    got = BF.as_f32(gold["out"], spec["dtype"])
    tol = 2.0 ** -7 * np.abs(ref) + 1e-2 if spec["dtype"] == "bf16" else 1e-4 * np.abs(ref) + 1e-4
    assert np.all(np.abs(got - ref) <= tol)


def test_e4m3_encoder_matches_torch():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.uniform(-448, 448, 20000), rng.normal(0, 1, 20000), rng.normal(0, 1e-2, 5000),
        np.arange(-480, 481) / 2.0 ** 6,                   # subnormal and tie neighbourhoods
        np.array([0.0, -0.0, 448.0, -448.0, 2.0 ** -9, 1.5 * 2.0 ** -9, 0.5 * 2.0 ** -9, 17.0, 19.0]),
    ]).astype(np.float32)
    vals = np.clip(vals, -448, 448)
    want = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(OF.e4m3_encode(vals), want)
    np.testing.assert_array_equal(OF.e4m3_decode(want), torch.from_numpy(want).view(
        torch.float8_e4m3fn).float().numpy())


def test_dropin_over_reference_functions(reference_root):
    import qwen3_8.fp8_linear as FL
    import qwen3_8.fp8_triton as FT

    from tokenfactory_b200 import fp8
    ours = inspect.signature(fp8.block_fp8_linear).parameters
    theirs = inspect.signature(FT.triton_block_fp8_linear).parameters
    assert list(ours) == list(theirs)
    ref_fn, ref_pred = FT.triton_block_fp8_linear, FT.can_use_triton_fp8_gemm
    fp8.install()
    try:
        assert FT.triton_block_fp8_linear is fp8.block_fp8_linear
        assert FL.triton_block_fp8_linear is fp8.block_fp8_linear
        assert FL.can_use_triton_fp8_gemm is fp8.can_use_block_fp8_gemm
        assert not fp8.can_use_block_fp8_gemm(torch.zeros(2, 16))  # CPU activations: not ours
    finally:
        fp8.uninstall()
    assert FT.triton_block_fp8_linear is ref_fn and FL.can_use_triton_fp8_gemm is ref_pred


def test_gemm_argument_checks_without_a_gpu():
    from tokenfactory_b200 import _capi
    lib = _capi.load()
    fake = 0x1000
    base = dict(q=fake, q_stride=256, x_scale=fake, w=fake, w_stride=256, w_scale=fake,
                ws_stride_n=2, ws_stride_k=1, block_h=128, block_w=128, out=fake, out_stride=128,
                out_dtype=1, M=4, N=128, K=256)
    a = _capi.FP8GemmArgs(**{**base, "block_w": 64})
    assert lib.tf_fp8_block_gemm(ctypes.byref(a), None) == _capi.TF_ERR_UNSUPPORTED
    a = _capi.FP8GemmArgs(**{**base, "K": 250, "q_stride": 256, "w_stride": 256})
    assert lib.tf_fp8_block_gemm(ctypes.byref(a), None) == _capi.TF_ERR_UNSUPPORTED
    a = _capi.FP8GemmArgs(**{**base, "q_stride": 264})
    assert lib.tf_fp8_block_gemm(ctypes.byref(a), None) == _capi.TF_ERR_ALIGNMENT
    a = _capi.FP8GemmArgs(**{**base, "x_scale": None})
    assert lib.tf_fp8_block_gemm(ctypes.byref(a), None) == _capi.TF_ERR_INVALID_ARG
    a = _capi.FP8GemmArgs(**{**base, "M": 0})
    assert lib.tf_fp8_block_gemm(ctypes.byref(a), None) == _capi.TF_OK
    qa = _capi.FP8QuantArgs(x=fake, x_stride=255, M=2, K=255, dtype=1, q=fake, x_scale=fake,
                            workspace=fake)
    assert lib.tf_fp8_quantize(ctypes.byref(qa), None) == _capi.TF_ERR_UNSUPPORTED
    qa = _capi.FP8QuantArgs(x=fake + 2, x_stride=256, M=2, K=256, dtype=1, q=fake, x_scale=fake,
                            workspace=fake)
    assert lib.tf_fp8_quantize(ctypes.byref(qa), None) == _capi.TF_ERR_ALIGNMENT
