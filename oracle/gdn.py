"""Oracle for the Gated DeltaNet (GDN) linear-attention hot path (TEST INFRASTRUCTURE; numpy).

Restates qwen3_8/linear_attention.py and qwen3_8/rms_norm_gated.py of yz29528/tokenFactory:
  causal_conv1d_step   - linear_attention.py:133-152   conv over [state | x], state roll, SiLU
  qk_prep / gates      - linear_attention.py:171-181   L2 norm, dk**-0.5, GVA expand, g and beta
  gated_delta_rule     - linear_attention.py:154-242   single step (:184-192) and chunk-64 WY
  batched_decode_step  - linear_attention.py:244-298
  rms_norm_gated       - rms_norm_gated.py:26-40
  linear_attention_core- linear_attention.py:300-363   dispatch + per-request loop + norm

Activations, conv_state and parameters are stored as `dtype` ("bf16" -> uint16 bit patterns,
"f32" -> float32); the recurrent state is float32 as in req_to_state_pool.py:90-103.  Every step
that the reference runs in the pool dtype is rounded to it here, every fp32 step stays fp32.
"""

from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import bf16 as _bf


def _silu(x: np.ndarray) -> np.ndarray:
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def _softplus(x: np.ndarray) -> np.ndarray:
    # torch.nn.functional.softplus with beta=1, threshold=20
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0)))).astype(np.float32)


def causal_conv1d_step(x: np.ndarray, conv_state: np.ndarray, weight: np.ndarray,
                       bias: Optional[np.ndarray], dtype: str) -> Tuple[np.ndarray, np.ndarray]:
    """Depthwise causal conv1d of one request's chunk (qwen3_8/linear_attention.py:133-152).

    x [E, C] and conv_state [C, K-1] are stored as `dtype`, weight [C, K] (Conv1d weight squeezed).
    padded = [state | x^T]; the new state is the last K-1 columns of padded (:142-143);
    out[t, c] = silu(sum_j w[c, j] * padded[c, t + j] + bias[c]), the conv result rounded to
    `dtype` and the SiLU result rounded again (both ops run on `dtype` tensors in the reference).
    Returns (out [E, C] as float32 values, new_state [C, K-1] in storage form).
    """
    e = x.shape[0]
    kk = weight.shape[1]
    xs = _bf.as_f32(x, dtype)
    st = _bf.as_f32(conv_state, dtype)
    w = _bf.as_f32(weight, dtype)
    padded = np.concatenate([st, xs.T], axis=1)  # [C, K-1+E]
    new_state = _bf.store(padded[:, -(kk - 1):], dtype) if kk > 1 else conv_state
    acc = np.zeros((xs.shape[1], e), dtype=np.float32)
    for j in range(kk):
        acc += w[:, j:j + 1] * padded[:, j:j + e]
    if bias is not None:
        acc += _bf.as_f32(bias, dtype)[:, None]
    conv = _bf.round_to(acc, dtype)
    out = _bf.round_to(_silu(conv), dtype)
    return out.T.copy(), new_state


def qk_prep(q: np.ndarray, k: np.ndarray, head_k_dim: int, v_per_k: int):
    """F.normalize(p=2, eps=1e-12) of q and k, q * dk**-0.5, repeat_interleave to v heads
    (qwen3_8/linear_attention.py:171-175).  q, k: float32 [E, Hk, dk] -> [E, Hv, dk]."""
    def _l2(x):
        n = np.sqrt(np.sum(x * x, axis=-1, keepdims=True, dtype=np.float32))
        return (x / np.maximum(n, np.float32(1e-12))).astype(np.float32)

    qn = _l2(q) * np.float32(head_k_dim ** -0.5)
    kn = _l2(k)
    return np.repeat(qn, v_per_k, axis=1), np.repeat(kn, v_per_k, axis=1)


def gates(a: np.ndarray, b: np.ndarray, A_log: np.ndarray, dt_bias: np.ndarray):
    """g = -exp(A_log) * softplus(a + dt_bias); beta = sigmoid(b)
    (qwen3_8/linear_attention.py:178-181).  All float32 values."""
    g = -np.exp(A_log.astype(np.float32)) * _softplus((a + dt_bias).astype(np.float32))
    beta = np.float32(1.0) / (np.float32(1.0) + np.exp(-b.astype(np.float32)))
    return g.astype(np.float32), beta.astype(np.float32)


def _solve_unit_lower(lhs: np.ndarray, rhs: np.ndarray) -> np.ndarray:
    """Forward substitution for unit lower-triangular lhs [H,C,C], rhs [H,C,V]
    (torch.linalg.solve_triangular(upper=False, unitriangular=True), :226-228)."""
    c = lhs.shape[1]
    u = np.zeros_like(rhs)
    for i in range(c):
        u[:, i] = rhs[:, i] - np.einsum("hj,hjv->hv", lhs[:, i, :i], u[:, :i])
    return u


def gated_delta_rule(q: np.ndarray, k: np.ndarray, v: np.ndarray, g: np.ndarray,
                     beta: np.ndarray, state: np.ndarray, chunk_size: int = 64) -> np.ndarray:
    """Gated delta rule over one request's tokens (qwen3_8/linear_attention.py:183-242).

    q, k [E, Hv, dk] (already normalised and GVA-expanded), v [E, Hv, dv], g/beta [E, Hv],
    state [Hv, dk, dv] float32 updated IN PLACE.  Returns o [E, Hv, dv] float32.
    E == 1 runs the single-step update (:184-192); E > 1 the chunk-wise WY form (:194-240).
    """
    e = q.shape[0]
    if e == 1:
        alpha = np.exp(g[0])[:, None, None]
        state *= alpha
        v_pred = np.einsum("hkd,hk->hd", state, k[0])
        delta = beta[0][:, None] * (v[0] - v_pred)
        state += np.einsum("hk,hd->hkd", k[0], delta)
        return np.einsum("hkd,hk->hd", state, q[0])[None].astype(np.float32)
    outs = []
    for s0 in range(0, e, chunk_size):
        s1 = min(s0 + chunk_size, e)
        c = s1 - s0
        qh = q[s0:s1].transpose(1, 0, 2)
        kh = k[s0:s1].transpose(1, 0, 2)
        vh = v[s0:s1].transpose(1, 0, 2)
        gh = g[s0:s1].T
        bh = beta[s0:s1].T
        gamma = np.cumsum(gh, axis=-1, dtype=np.float32)
        diff = gamma[:, :, None] - gamma[:, None, :]
        tril = np.tril(np.ones((c, c), dtype=bool))
        stril = np.tril(np.ones((c, c), dtype=bool), k=-1)
        gamma_tril = np.exp(np.where(tril, diff, -np.inf)).astype(np.float32)
        gamma_stril = np.where(stril, gamma_tril, 0.0).astype(np.float32)
        kk = kh @ kh.transpose(0, 2, 1)
        lhs = np.eye(c, dtype=np.float32)[None] + bh[:, :, None] * gamma_stril * kk
        exp_gamma = np.exp(gamma)[:, :, None]
        k_state = kh @ state
        rhs = bh[:, :, None] * (vh - exp_gamma * k_state)
        u = _solve_unit_lower(lhs, rhs)
        q_state = qh @ state
        qk = qh @ kh.transpose(0, 2, 1)
        out_h = exp_gamma * q_state + (gamma_tril * qk) @ u
        outs.append(out_h.transpose(1, 0, 2))
        total = np.exp(gamma[:, -1])[:, None, None]
        to_end = np.exp(gamma[:, -1:] - gamma)[:, :, None]
        state *= total
        state += (kh * to_end).transpose(0, 2, 1) @ u
    return np.concatenate(outs, axis=0).astype(np.float32)


def split_conv_out(conv_out: np.ndarray, nk: int, nv: int, dk: int, dv: int):
    """conv_out [E, conv_dim] -> q, k [E, Hk, dk], v [E, Hv, dv] (:271-276, :347-353)."""
    e = conv_out.shape[0]
    key_dim = nk * dk
    q = conv_out[:, :key_dim].reshape(e, nk, dk)
    k = conv_out[:, key_dim:2 * key_dim].reshape(e, nk, dk)
    v = conv_out[:, 2 * key_dim:].reshape(e, nv, dv)
    return q, k, v


def rms_norm_gated(x: np.ndarray, z: np.ndarray, weight: np.ndarray, head_dim: int,
                   eps: float, dtype: str) -> np.ndarray:
    """w * x/rms(x per head) * silu(z) in float32, rounded to `dtype`
    (qwen3_8/rms_norm_gated.py:26-40).  x, z, weight float32 values; weight has either one entry per
    channel or `head_dim` entries shared by every head; returns float32 values of `dtype`."""
    t, c = x.shape
    xh = x.reshape(t, c // head_dim, head_dim).astype(np.float32)
    var = np.mean(xh * xh, axis=-1, keepdims=True, dtype=np.float32)
    xn = (xh / np.sqrt(var + np.float32(eps))).reshape(t, c)
    w = weight.astype(np.float32)
    if w.shape[0] != c:
        w = np.tile(w, c // w.shape[0])
    return _bf.round_to((w * xn * _silu(z.astype(np.float32))).astype(np.float32), dtype)


def linear_attention_core(qkv: np.ndarray, b: np.ndarray, a: np.ndarray, z: Optional[np.ndarray],
                          params: Dict[str, np.ndarray], conv_state: np.ndarray,
                          ssm_state: np.ndarray, req_pool_indices: Sequence[int],
                          extend_lens: Sequence[int], dims: Dict[str, int], dtype: str,
                          norm_eps: float = 1e-6) -> np.ndarray:
    """Linear-attention forward between the projections and out_proj
    (qwen3_8/linear_attention.py:300-363).

    qkv [T, conv_dim], b/a [T, Hv], z [T, Hv*dv] stored as `dtype`; conv_state [slots, C, K-1]
    (storage form) and ssm_state [slots, Hv, dk, dv] float32 are updated IN PLACE at the request
    rows.  params: conv_weight [C, K], conv_bias or None, A_log [Hv], dt_bias [Hv], norm_weight.
    Returns float32 values of `dtype`: the normed output if z is given, else the raw GDN output.

    Every request runs conv + gated delta rule in turn, as the reference does for extend/mixed
    batches (:337-358); an all-decode batch (:316-326) gives the same numbers because the batched
    decode step and the single-step branch are the same arithmetic.
    """
    nk, nv, dk, dv = dims["num_k_heads"], dims["num_v_heads"], dims["head_k_dim"], dims["head_v_dim"]
    vpk = nv // nk
    A_log = _bf.as_f32(params["A_log"], dtype)
    dt_bias = _bf.as_f32(params["dt_bias"], dtype)
    outs: List[np.ndarray] = []
    t0 = 0
    for i, ext in enumerate(int(x) for x in extend_lens):
        r = int(req_pool_indices[i])
        conv_out, new_state = causal_conv1d_step(qkv[t0:t0 + ext], conv_state[r],
                                                 params["conv_weight"], params.get("conv_bias"),
                                                 dtype)
        conv_state[r] = new_state
        q, k, v = split_conv_out(conv_out, nk, nv, dk, dv)
        qe, ke = qk_prep(q, k, dk, vpk)
        g, beta = gates(_bf.as_f32(a[t0:t0 + ext], dtype), _bf.as_f32(b[t0:t0 + ext], dtype),
                        A_log, dt_bias)
        st = ssm_state[r]
        o = gated_delta_rule(qe, ke, v.astype(np.float32), g, beta, st)
        ssm_state[r] = st
        outs.append(_bf.round_to(o.reshape(ext, nv * dv), dtype))
        t0 += ext
    out = np.concatenate(outs, axis=0) if outs else np.zeros((0, nv * dv), np.float32)
    if z is None:
        return out
    return rms_norm_gated(out, _bf.as_f32(z, dtype), _bf.as_f32(params["norm_weight"], dtype),
                          dv, norm_eps, dtype)


def batched_decode_step(qkv: np.ndarray, b: np.ndarray, a: np.ndarray,
                        params: Dict[str, np.ndarray], conv_state: np.ndarray,
                        ssm_state: np.ndarray, req_pool_indices: Sequence[int],
                        dims: Dict[str, int], dtype: str) -> np.ndarray:
    """Batched one-token step (qwen3_8/linear_attention.py:244-298); returns float32 values of
    `dtype` [B, Hv*dv] and updates the states in place."""
    return linear_attention_core(qkv, b, a, None, params, conv_state, ssm_state,
                                 req_pool_indices, [1] * len(req_pool_indices), dims, dtype)
