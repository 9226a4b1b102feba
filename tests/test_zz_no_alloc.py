"""The allocation-free paged-decode entry point, tf_paged_decode_attn_noalloc.

Callers that cannot allocate device memory themselves - a host runtime that binds this C ABI
through a plain FFI and has no CUDA allocator of its own, or a serving process that gives all free
device memory to its own pool at start-up - use this entry point instead of tf_paged_decode_attn:
it takes the same inputs and outputs but keeps its scratch in a fixed array inside the library, so
it needs no workspace.  This test calls it through the C ABI twice in a row, on two different
batches (the second call finds the first call's leftovers in the shared scratch), and checks each
result against the workspace entry point within the hot path's bf16 tolerance.  It also checks
that a batch too large for the fixed scratch is refused with a clear error instead of running, and
that a call captured into a CUDA graph (after a first call outside capture) replays correctly.
"""

import ctypes

import numpy as np
import pytest

from tests.golden import cases as C
from tests.helpers import assert_close, to_torch, values

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _batch(seed, B, hq, hkv, d, lmax):
    rng = np.random.default_rng(seed)
    seq = [int(x) for x in rng.integers(1, lmax + 1, B)]
    spec = dict(dtype="bf16", hq=hq, hkv=hkv, d=d, seq=seq, ext=[1] * B,
                req=[int(x) for x in rng.permutation(B + 2)[:B]], slots=sum(seq) + 9,
                rows=B + 2, cols=lmax + 4, seed=seed)
    inp = C.attn_inputs(spec)
    return spec, {k: to_torch(v, "bf16") for k, v in inp.items()}


def _noalloc(spec, t, out):
    from tokenfactory_b200 import _capi, ops
    args, keep = ops._paged_args(t["q"], t["k_buf"], t["v_buf"], t["req_to_token"],
                                 t["req_pool_indices"], t["seq_lens"], None, spec["d"] ** -0.5,
                                 t["gate"], "sigmoid", out, max(spec["seq"]), 1, "clamp", None)
    lib = _capi.load()
    st = lib.tf_paged_decode_attn_noalloc(ctypes.byref(args),
                                          torch.cuda.current_stream().cuda_stream)
    _capi.check("tf_paged_decode_attn_noalloc", st)
    del keep


def test_noalloc_decode_matches_workspace_entry_point_on_two_calls():
    from tokenfactory_b200 import ops
    for seed, shape in ((1, (24, 32, 4, 256, 3000)), (2, (9, 16, 2, 256, 9000))):
        B, hq, hkv, d, lmax = shape
        spec, t = _batch(seed, B, hq, hkv, d, lmax)
        want = ops.paged_decode(t["q"], t["k_buf"], t["v_buf"], t["req_to_token"],
                                t["req_pool_indices"], t["seq_lens"], d ** -0.5, max(spec["seq"]),
                                gate=t["gate"], gate_mode="sigmoid")
        got = torch.full_like(want, float("nan"))
        _noalloc(spec, t, got)
        torch.cuda.synchronize()
        assert_close(values(got, "bf16"), values(want, "bf16"), "bf16",
                     what=f"noalloc call {seed}")


def test_noalloc_call_replays_inside_a_cuda_graph():
    """After one call outside capture has resolved the scratch's device address, a call captured
    into a CUDA graph replays with the same result as the workspace entry point."""
    from tokenfactory_b200 import ops
    spec, t = _batch(3, 17, 32, 4, 256, 4000)
    want = ops.paged_decode(t["q"], t["k_buf"], t["v_buf"], t["req_to_token"],
                            t["req_pool_indices"], t["seq_lens"], 256 ** -0.5, max(spec["seq"]),
                            gate=t["gate"], gate_mode="sigmoid")
    got = torch.full_like(want, float("nan"))
    _noalloc(spec, t, got)  # outside capture: resolves the scratch address on this device
    torch.cuda.synchronize()
    got.fill_(float("nan"))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _noalloc(spec, t, got)
    for _ in range(2):
        got.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert_close(values(got, "bf16"), values(want, "bf16"), "bf16", what="noalloc replay")
    del graph


def test_noalloc_refuses_a_batch_beyond_its_fixed_scratch():
    """The fixed scratch serves batches of up to 32768 requests; a batch of 60,000 is rejected
    before any launch (the arguments below point at a tiny pool and are never read)."""
    from tokenfactory_b200 import _capi
    dummy = torch.zeros(64, dtype=torch.int64, device="cuda")
    pool = torch.zeros((4, 1, 256), dtype=torch.bfloat16, device="cuda")
    big = 60_000
    a = _capi.PagedAttnArgs(
        q=pool.data_ptr(), q_stride_tok=8 * 256, q_stride_head=256,
        k_buffer=pool.data_ptr(), v_buffer=pool.data_ptr(), kv_stride_slot=256,
        kv_stride_head=256, num_slots=4, req_to_token=dummy.data_ptr(), r2t_stride=8,
        r2t_rows=8, r2t_cols=8, req_pool_indices=dummy.data_ptr(), seq_lens=dummy.data_ptr(),
        out=pool.data_ptr(), out_stride_tok=8 * 256, out_stride_head=256, batch_size=big,
        num_tokens=big, num_q_heads=8, num_kv_heads=1, head_dim=256, max_seq_len=1,
        max_extend_len=1, scale=0.0625, dtype=_capi.TF_DTYPE_BF16,
        gate_mode=_capi.TF_GATE_NONE, slot_mode=_capi.TF_SLOT_CLAMP)
    lib = _capi.load()
    st = lib.tf_paged_decode_attn_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert st == _capi.TF_ERR_WORKSPACE
    assert b"built-in scratch" in lib.tf_last_error()
