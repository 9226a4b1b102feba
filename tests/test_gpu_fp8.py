"""GPU parity of the block-FP8 linear (tf_fp8_quantize + tf_fp8_block_gemm) through the C ABI.

Activation quantization is bit-exact with the reference's recorded arguments; the output is
within one bf16 step (2^-7 relative) plus 1e-2 of the reference kernel's output, and of the
float64 oracle at larger shapes (tiles with row and column tails, ragged last K block, bias,
decode-sized M, per-tensor scale)."""

import numpy as np
import pytest

from oracle import bf16 as BF
from oracle import fp8 as OF
from tests.golden import cases as C
from tests.golden.load import fp8_case
from tests.helpers import to_numpy, to_torch

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _tensors(inp, dt):
    x = to_torch(inp["x"], dt)
    w = torch.from_numpy(inp["w"].copy()).cuda().view(torch.float8_e4m3fn)
    ws = torch.from_numpy(inp["w_scale"]).cuda() if "w_scale" in inp else None
    bias = to_torch(inp["bias"], dt) if "bias" in inp else None
    return x, w, ws, bias


def _tol(ref, dt):
    return 2.0 ** -7 * np.abs(ref) + 1e-2 if dt == "bf16" else 1e-4 * np.abs(ref) + 1e-4


@pytest.mark.parametrize("name", sorted(C.FP8_CASES))
def test_matches_reference_kernel_fixture(name):
    from tokenfactory_b200 import ops
    spec, inp, gold = fp8_case(name)
    dt = spec["dtype"]
    x, w, ws, bias = _tensors(inp, dt)
    q, s = ops.fp8_quantize(x)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), gold["q"])
    assert float(s.item()) == float(gold["x_scale"][0])
    out = ops.block_fp8_linear(x, w, ws, bias)
    got = BF.as_f32(to_numpy(out), dt)
    ref = BF.as_f32(gold["out"], dt)
    assert np.all(np.abs(got - ref) <= _tol(ref, dt) + 2.0 ** -7 * np.abs(ref)), name


@pytest.mark.parametrize("M,N,K,scales,bias", [(300, 1000, 2048, True, True), (1, 512, 1024, True, False),
                                               (129, 384, 400, True, False), (64, 256, 512, False, True)])
def test_larger_shapes_match_oracle(M, N, K, scales, bias):
    from tokenfactory_b200 import ops
    spec = dict(dtype="bf16", M=M, N=N, K=K, scales=scales, bias=bias, seed=M + N + K)
    inp = C.fp8_inputs(spec)
    x, w, ws, b = _tensors(inp, "bf16")
    out = ops.block_fp8_linear(x.view(M, K), w, ws, b)
    q, s = ops.fp8_quantize(x)
    torch.cuda.synchronize()
    qn, sn = OF.quantize_act(inp["x"], "bf16")
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), qn)
    ref = OF.block_fp8_linear(qn, sn, inp["w"], inp.get("w_scale"),
                              BF.as_f32(inp["bias"], "bf16") if bias else None)
    got = BF.as_f32(to_numpy(out), "bf16")
    assert np.all(np.abs(got - ref) <= _tol(ref, "bf16")), np.abs(got - ref).max()


@pytest.mark.parametrize("M,N,K,scales,bias", [(1100, 4400, 1008, True, True),
                                               (2048, 4352, 512, True, False),
                                               (1300, 4608, 256, False, True)])
def test_wide_tiles_match_oracle(M, N, K, scales, bias):
    """Problems with at least one 128 x 256 tile per SM take the persistent wide-tile kernel:
    row and column tails (a 256-column tile whose second half lies past N), a ragged last K block,
    more tiles than SMs (CTAs that walk several tiles through one stage ring), and both halves of
    a tile with their own weight-scale rows."""
    from tokenfactory_b200 import ops
    tiles = -(-M // 128) * -(-N // 256)
    assert tiles >= torch.cuda.get_device_properties(0).multi_processor_count
    spec = dict(dtype="bf16", M=M, N=N, K=K, scales=scales, bias=bias, seed=M + N + K)
    inp = C.fp8_inputs(spec)
    x, w, ws, b = _tensors(inp, "bf16")
    out = ops.block_fp8_linear(x.view(M, K), w, ws, b)
    torch.cuda.synchronize()
    qn, sn = OF.quantize_act(inp["x"], "bf16")
    ref = OF.block_fp8_linear(qn, sn, inp["w"], inp.get("w_scale"),
                              BF.as_f32(inp["bias"], "bf16") if bias else None)
    got = BF.as_f32(to_numpy(out), "bf16")
    assert np.all(np.abs(got - ref) <= _tol(ref, "bf16")), np.abs(got - ref).max()
