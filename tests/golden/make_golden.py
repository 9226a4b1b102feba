"""Generate the golden vectors of the hot path by running the REFERENCE's own torch functions.

    python tests/golden/make_golden.py --reference <path to a yz29528/tokenFactory checkout>

Needs the reference's Python package importable on the CPU (torch only); writes
tests/golden/*_golden.npz.  Inputs come from
tests/golden/cases.py (seeded numpy), so the fixtures store outputs and an input checksum only.

Reference functions exercised (paths inside the reference project):
  Qwen3_8FullAttention._slot_based_attention   qwen3_8/full_attention.py:163-283
  output gate attn * F.silu(gate)              qwen3_8/full_attention.py:157-158
  Qwen3_8LinearAttention._batched_decode_step  qwen3_8/linear_attention.py:244-298
  Qwen3_8LinearAttention._causal_conv1d_step   qwen3_8/linear_attention.py:133-152
  Qwen3_8LinearAttention._gated_delta_rule_step qwen3_8/linear_attention.py:154-242
  the extend loop of forward()                 qwen3_8/linear_attention.py:329-358
  Qwen3_8RMSNormGated.forward                  qwen3_8/rms_norm_gated.py:26-40
  Qwen3_8FullAttention.forward                 qwen3_8/full_attention.py:112-161
  Qwen3_8LinearAttention.forward               qwen3_8/linear_attention.py:300-364
  Qwen3_8RMSNorm.forward (q_norm / k_norm)     qwen3_8/rms_norm.py:19-24
  PartialRotaryEmbedding.forward               qwen3_8/rotary_embedding.py:46-95
  the pool write of Qwen3_8FullAttention       qwen3_8/full_attention.py:147-149
  ReqToStatePool snapshot calls                req_to_state_pool.py:34-194
  ModelRunner._prepare_forward_batch           engine/model_runner.py:108-188
  triton_block_fp8_linear (Triton interpreter) qwen3_8/fp8_triton.py:17-181
"""

import argparse
import os
import sys

# the reference's block-FP8 kernel is a Triton kernel: on this CPU-only host it runs in Triton's
# interpreter (set before anything imports triton)
os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden import cases as C  # noqa: E402


# the gated outputs are recorded for the smaller cases only, to keep the fixtures small
GATED_MAX_ELEMS = 40000


def _t(x: np.ndarray, dtype: str) -> torch.Tensor:
    """numpy storage (uint16 bits for bf16) -> torch tensor of the case dtype."""
    if dtype == "bf16" and x.dtype == np.uint16:
        return torch.from_numpy(x.view(np.int16).copy()).view(torch.bfloat16)
    if x.dtype == np.int64:
        return torch.from_numpy(x.copy())
    return torch.from_numpy(np.asarray(x, np.float32).copy())


def _np(x: torch.Tensor) -> np.ndarray:
    """torch tensor -> numpy storage (bf16 -> uint16 bits)."""
    x = x.detach().contiguous()
    if x.dtype == torch.bfloat16:
        return x.view(torch.int16).numpy().view(np.uint16).copy()
    return x.numpy().copy()


def _tdt(dtype: str):
    return torch.bfloat16 if dtype == "bf16" else torch.float32


def attention_golden(ref) -> dict:
    from qwen3_8 import ForwardBatch, Qwen3_8Config
    from qwen3_8.full_attention import Qwen3_8FullAttention

    out = {}
    for name, spec in C.ATTN_CASES.items():
        inp = C.attn_inputs(spec)
        dt = spec["dtype"]
        cfg = Qwen3_8Config(hidden_size=64, intermediate_size=64, num_hidden_layers=1,
                            layer_types=["full_attention"], num_attention_heads=spec["hq"],
                            num_key_value_heads=spec["hkv"], head_dim=spec["d"])
        fa = Qwen3_8FullAttention(cfg, 0).eval()
        q = _t(inp["q"], dt)
        kb, vb = _t(inp["k_buf"], dt), _t(inp["v_buf"], dt)
        seq, ext = spec["seq"], spec["ext"]
        fb = ForwardBatch(batch_size=len(seq), req_pool_indices=_t(inp["req_pool_indices"], dt),
                          seq_lens=_t(inp["seq_lens"], dt),
                          prefix_lens=_t(inp["seq_lens"] - inp["extend_lens"], dt),
                          extend_lens=list(ext), out_cache_loc=_t(inp["out_cache_loc"], dt),
                          req_to_token=_t(inp["req_to_token"], dt), is_prefill=max(ext) > 1,
                          max_seq_len=max(seq), max_extend_len=max(ext),
                          extend_lens_tensor=_t(inp["extend_lens"], dt),
                          req_pool_indices_list=list(spec["req"]))
        with torch.inference_mode():
            attn = fa._slot_based_attention(q, kb, vb, fb)
            t = attn.shape[0]
            flat = attn.reshape(t, spec["hq"] * spec["d"])
            gate = _t(inp["gate"], dt).reshape(t, -1)
            silu = flat * F.silu(gate)
            sig = flat * torch.sigmoid(gate)
        out[f"{name}/out"] = _np(attn)
        if attn.numel() <= GATED_MAX_ELEMS:
            out[f"{name}/out_silu"] = _np(silu)
            out[f"{name}/out_sigmoid"] = _np(sig)
        out[f"{name}/checksum"] = np.frombuffer(C.checksum(inp).encode(), dtype=np.uint8)
    return out


def gdn_golden(ref) -> dict:
    from qwen3_8 import Qwen3_8Config
    from qwen3_8.linear_attention import Qwen3_8LinearAttention

    out = {}
    for name, spec in C.GDN_CASES.items():
        inp = C.gdn_inputs(spec)
        dt = spec["dtype"]
        tdt = _tdt(dt)
        cfg = Qwen3_8Config(hidden_size=64, intermediate_size=64, num_hidden_layers=1,
                            layer_types=["linear_attention"],
                            linear_num_key_heads=spec["nk"], linear_num_value_heads=spec["nv"],
                            linear_key_head_dim=spec["dk"], linear_value_head_dim=spec["dv"],
                            linear_conv_kernel_dim=spec["kc"])
        la = Qwen3_8LinearAttention(cfg, 0).eval().to(tdt)
        with torch.no_grad():
            la.conv1d.weight.copy_(_t(inp["conv_weight"], dt).unsqueeze(1))
            la.A_log.copy_(_t(inp["A_log"], dt))
            la.dt_bias.copy_(_t(inp["dt_bias"], dt))
            la.norm.weight.copy_(_t(inp["norm_weight"], dt))
        qkv, b, a, z = (_t(inp[k], dt) for k in ("qkv", "b", "a", "z"))
        conv_state = _t(inp["conv_state"], dt)
        ssm_state = torch.from_numpy(inp["ssm_state"].copy())
        req = spec["req"]
        ext = spec["ext"]
        with torch.inference_mode():
            if all(e == 1 for e in ext):
                raw = la._batched_decode_step(qkv, b, a, conv_state, ssm_state,
                                              torch.tensor(req, dtype=torch.long))
            else:
                outs, off = [], 0
                for i, e in enumerate(ext):
                    r = req[i]
                    co = la._causal_conv1d_step(qkv[off:off + e], conv_state[r])
                    qi, ki, vi = co.split([la.key_dim, la.key_dim, la.value_dim], dim=-1)
                    oi = la._gated_delta_rule_step(
                        qi.reshape(e, la.num_k_heads, la.head_k_dim),
                        ki.reshape(e, la.num_k_heads, la.head_k_dim),
                        vi.reshape(e, la.num_v_heads, la.head_v_dim),
                        b[off:off + e], a[off:off + e], ssm_state[r])
                    outs.append(oi.reshape(e, la.value_dim))
                    off += e
                raw = torch.cat(outs, dim=0)
            normed = la.norm(raw, z)
        out[f"{name}/raw"] = _np(raw)
        out[f"{name}/normed"] = _np(normed)
        out[f"{name}/conv_state"] = _np(conv_state[req])
        out[f"{name}/ssm_state"] = _np(ssm_state[req])
        out[f"{name}/checksum"] = np.frombuffer(C.checksum(inp).encode(), dtype=np.uint8)
    return out


class _Pool:
    """The two cache-pool views the attention forwards read (qwen3_8/hybrid_cache_pool.py:151-158)."""

    def __init__(self, k_buf=None, v_buf=None, conv_state=None, ssm_state=None):
        self.k, self.v, self.c, self.s = k_buf, v_buf, conv_state, ssm_state

    def get_full_kv_buffers(self, layer_idx):
        return self.k, self.v

    def get_linear_states(self, layer_idx):
        return self.c, self.s


def module_golden(ref) -> dict:
    from qwen3_8 import ForwardBatch, Qwen3_8Config
    from qwen3_8.full_attention import Qwen3_8FullAttention
    from qwen3_8.linear_attention import Qwen3_8LinearAttention

    m = C.MODULE_DIMS
    cfg = Qwen3_8Config(hidden_size=m["hidden"], intermediate_size=64, num_hidden_layers=4,
                        layer_types=["linear_attention"] * 3 + ["full_attention"],
                        num_attention_heads=m["hq"], num_key_value_heads=m["hkv"],
                        head_dim=m["d"], linear_num_key_heads=m["nk"],
                        linear_num_value_heads=m["nv"], linear_key_head_dim=m["dk"],
                        linear_value_head_dim=m["dv"], linear_conv_kernel_dim=m["kc"])
    out = {}
    for name, spec in C.MODULE_CASES.items():
        dt = _tdt(spec["dtype"])
        w = C.module_weights(spec)
        inp = C.module_inputs(spec)
        out[f"{name}/checksum"] = np.frombuffer(
            C.checksum({**w, **inp}).encode(), dtype=np.uint8)
        inp = {k: v.copy() for k, v in inp.items()}  # the forward writes the pools in place
        mod = (Qwen3_8FullAttention(cfg, 3) if spec["kind"] == "full"
               else Qwen3_8LinearAttention(cfg, 0))
        mod.load_state_dict({k: torch.from_numpy(v) for k, v in w.items()}, strict=False)
        mod = mod.eval().to(dt)
        hidden = torch.from_numpy(inp["hidden"]).to(dt)
        ext = spec["ext"]
        T = int(sum(ext))
        with torch.inference_mode():
            if spec["kind"] == "full":
                kb = torch.from_numpy(inp["k_buf"]).to(dt)
                vb = torch.from_numpy(inp["v_buf"]).to(dt)
                pool = _Pool(kb, vb)
                fb = ForwardBatch(batch_size=len(ext),
                                  req_pool_indices=torch.from_numpy(inp["req_pool_indices"]),
                                  seq_lens=torch.from_numpy(inp["seq_lens"]),
                                  prefix_lens=torch.from_numpy(inp["seq_lens"] - inp["extend_lens"]),
                                  extend_lens=list(ext),
                                  out_cache_loc=torch.from_numpy(inp["out_cache_loc"]),
                                  req_to_token=torch.from_numpy(inp["req_to_token"]),
                                  is_prefill=max(ext) > 1)
                y = mod(hidden, torch.from_numpy(inp["positions"]), pool, fb)
                loc = torch.from_numpy(inp["out_cache_loc"])
                out[f"{name}/k_rows"] = _np(kb[loc])
                out[f"{name}/v_rows"] = _np(vb[loc])
            else:
                cs = torch.from_numpy(inp["conv_state"]).to(dt)
                ss = torch.from_numpy(inp["ssm_state"].copy())
                pool = _Pool(conv_state=cs, ssm_state=ss)
                fb = ForwardBatch(batch_size=len(ext),
                                  req_pool_indices=torch.from_numpy(inp["req_pool_indices"]),
                                  seq_lens=torch.from_numpy(inp["extend_lens"] + 5),
                                  prefix_lens=torch.full((len(ext),), 5, dtype=torch.long),
                                  extend_lens=list(ext),
                                  out_cache_loc=torch.zeros(T, dtype=torch.long),
                                  req_to_token=torch.zeros((1, 1), dtype=torch.long),
                                  is_prefill=max(ext) > 1)
                y = mod(hidden, pool, fb)
                out[f"{name}/conv_state"] = _np(cs)
                out[f"{name}/ssm_state"] = _np(ss)
        out[f"{name}/out"] = _np(y)
    return out


def prologue_golden(ref) -> dict:
    """q/k RMSNorm, partial (M-)RoPE and the pool write, through the reference's own modules
    (the steps of Qwen3_8FullAttention.forward, qwen3_8/full_attention.py:142-149)."""
    from qwen3_8.rms_norm import Qwen3_8RMSNorm
    from qwen3_8.rotary_embedding import PartialRotaryEmbedding

    out = {}
    for name, spec in C.PROLOGUE_CASES.items():
        inp = C.prologue_inputs(spec)
        dt, d = spec["dtype"], spec["d"]
        sec, inter = spec["mrope"] if spec["mrope"] else ([11, 11, 10], True)
        qn, kn = Qwen3_8RMSNorm(d, eps=C.PROLOGUE_EPS), Qwen3_8RMSNorm(d, eps=C.PROLOGUE_EPS)
        rope = PartialRotaryEmbedding(head_dim=d, partial_rotary_factor=0.25,
                                      rope_theta=C.PROLOGUE_THETA, mrope_section=list(sec),
                                      mrope_interleaved=inter)
        with torch.inference_mode():
            qn.weight.copy_(_t(inp["q_norm_weight"], dt).float())
            kn.weight.copy_(_t(inp["k_norm_weight"], dt).float())
            q = _t(C.prologue_q(inp, spec), dt)
            k, v = _t(inp["k"], dt), _t(inp["v"], dt)
            q, k = rope(qn(q), kn(k), torch.from_numpy(inp["positions"]))
            kb, vb = _t(inp["k_buf"], dt), _t(inp["v_buf"], dt)
            loc = torch.from_numpy(inp["out_cache_loc"])
            kb[loc] = k
            vb[loc] = v
        out[f"{name}/q_out"] = _np(q)
        out[f"{name}/k_buf"] = _np(kb)
        out[f"{name}/v_buf"] = _np(vb)
        out[f"{name}/inv_freq"] = rope.inv_freq.numpy().astype(np.float32)
        out[f"{name}/checksum"] = np.frombuffer(C.checksum(inp).encode(), dtype=np.uint8)
    return out


def state_pool_golden(ref) -> dict:
    """ReqToStatePool built from a Qwen3_8Config, its tensors filled with the case's values, then
    STATE_POOL_SCRIPT applied through the reference's own methods (req_to_state_pool.py:34-194)."""
    from qwen3_8 import Qwen3_8Config
    from req_to_state_pool import ReqToStatePool

    from oracle.state_pool import bookkeeping, run_script

    out = {}
    for name, spec in C.STATE_POOL_CASES.items():
        inp = C.state_pool_inputs(spec)
        cfg = Qwen3_8Config(num_hidden_layers=spec["layers"] + 1,
                            layer_types=["linear_attention"] * spec["layers"] + ["full_attention"],
                            linear_num_key_heads=spec["nk"], linear_num_value_heads=spec["nv"],
                            linear_key_head_dim=spec["dk"], linear_value_head_dim=spec["dv"],
                            linear_conv_kernel_dim=spec["kc"])
        pool = ReqToStatePool(spec["max_reqs"], spec["max_snapshots"], config=cfg, device="cpu",
                              dtype=_tdt(spec["dtype"]))
        assert tuple(pool.conv_state.shape) == inp["conv_state"].shape
        assert tuple(pool.ssm_state.shape) == inp["ssm_state"].shape
        with torch.inference_mode():
            pool.conv_state.copy_(_t(inp["conv_state"], spec["dtype"]))
            pool.ssm_state.copy_(_t(inp["ssm_state"], "f32"))
        allocs = run_script(pool, C.STATE_POOL_SCRIPT)
        free, occ, tags = bookkeeping(pool)
        out[f"{name}/conv_state"] = _np(pool.conv_state)
        out[f"{name}/ssm_state"] = _np(pool.ssm_state)
        out[f"{name}/allocs"] = np.asarray([-1 if a is None else a for a in allocs], np.int64)
        out[f"{name}/free_slots"] = np.asarray(free, np.int64)
        out[f"{name}/occupied"] = np.asarray(occ, np.bool_)
        out[f"{name}/tags"] = np.asarray(tags)
        out[f"{name}/checksum"] = np.frombuffer(C.checksum(inp).encode(), dtype=np.uint8)
    return out


def runner_golden(ref) -> dict:
    """ModelRunner._prepare_forward_batch of the reference, run as an unbound method on a stand-in
    holding the attributes it reads (device, req_to_token_tensor, _req_synced_lens)."""
    from types import SimpleNamespace

    from engine.model_runner import ModelRunner

    case = C.RUNNER_CASE
    me = SimpleNamespace(device="cpu", _req_synced_lens=[0] * case["max_reqs"],
                         req_to_token_tensor=torch.full((case["max_reqs"], case["max_ctx"]), -1,
                                                        dtype=torch.long))
    out = {}
    for i, (reqs, table, dirty) in enumerate(C.runner_script(case)):
        objs = [SimpleNamespace(**r) for r in reqs]
        d = None if dirty is None else list(dirty)
        ids, pos, fb = ModelRunner._prepare_forward_batch(me, objs, table, d)
        out[f"step{i}/input_ids"] = ids.numpy()
        out[f"step{i}/positions"] = pos.numpy()
        out[f"step{i}/out_cache_loc"] = fb.out_cache_loc.numpy()
        out[f"step{i}/req_pool_indices"] = fb.req_pool_indices.numpy()
        out[f"step{i}/seq_lens"] = fb.seq_lens.numpy()
        out[f"step{i}/prefix_lens"] = fb.prefix_lens.numpy()
        out[f"step{i}/extend_lens"] = fb.extend_lens_tensor.numpy()
        out[f"step{i}/meta"] = np.asarray([fb.batch_size, int(fb.is_prefill), fb.max_seq_len,
                                           fb.max_extend_len], np.int64)
        out[f"step{i}/req_to_token"] = me.req_to_token_tensor.numpy().copy()
        out[f"step{i}/synced_lens"] = np.asarray(me._req_synced_lens, np.int64)
        if d is not None:
            out[f"step{i}/dirty_from"] = np.asarray(d, np.int64)
    return out


def fp8_golden(ref) -> dict:
    """triton_block_fp8_linear of the reference (its torch quantization lines and its Triton
    kernel, interpreted) on CPU tensors; the quantized activations and scale are the arguments
    the wrapper hands its kernel, recorded on the way through."""
    import qwen3_8.fp8_triton as F8

    real = F8._block_fp8_gemm_kernel
    seen = {}

    class Recorder:  # the launch `kernel[grid](x_fp8, w, out, x_scale, ...)`, recorded
        def __getitem__(self, grid):
            def launch(*args, **kw):
                seen["q"], seen["x_scale"] = args[0].clone(), args[3].clone()
                return real[grid](*args, **kw)
            return launch

    F8._block_fp8_gemm_kernel = Recorder()
    out = {}
    try:
        for name, spec in C.FP8_CASES.items():
            inp = C.fp8_inputs(spec)
            dt = spec["dtype"]
            x = _t(inp["x"], dt)
            w = torch.from_numpy(inp["w"].copy()).view(torch.float8_e4m3fn)
            ws = torch.from_numpy(inp["w_scale"]) if "w_scale" in inp else None
            bias = _t(inp["bias"], dt) if "bias" in inp else None
            y = F8.triton_block_fp8_linear(x, w, ws, bias, 128, 128)
            out[f"{name}/out"] = _np(y)
            out[f"{name}/q"] = seen["q"].view(torch.uint8).numpy().copy()
            out[f"{name}/x_scale"] = seen["x_scale"].reshape(1).numpy().astype(np.float32)
            out[f"{name}/checksum"] = np.frombuffer(C.checksum(inp).encode(), dtype=np.uint8)
    finally:
        F8._block_fp8_gemm_kernel = real
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", required=True,
                    help="root of a yz29528/tokenFactory checkout (its qwen3_8 package)")
    ap.add_argument("--only", nargs="*", default=None,
                    help="fixture names to regenerate (attention gdn module prologue state_pool runner fp8)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    torch.manual_seed(0)
    makers = dict(attention=attention_golden, gdn=gdn_golden, module=module_golden,
                  prologue=prologue_golden, state_pool=state_pool_golden,
                  runner=runner_golden, fp8=fp8_golden)
    for name, make in makers.items():
        if args.only is not None and name not in args.only:
            continue
        f = os.path.join(HERE, f"{name}_golden.npz")
        np.savez_compressed(f, **make(args))
        print(os.path.basename(f), os.path.getsize(f), "bytes")


if __name__ == "__main__":
    main()
