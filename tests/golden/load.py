"""Load the committed golden vectors and regenerate their inputs (see make_golden.py)."""

import os

import numpy as np

from . import cases as C

HERE = os.path.dirname(os.path.abspath(__file__))
_CACHE = {}


def _npz(name: str):
    if name not in _CACHE:
        _CACHE[name] = np.load(os.path.join(HERE, name))
    return _CACHE[name]


def attention_case(name: str):
    """(spec, inputs, golden outputs) of an attention case; asserts the inputs match the ones the
    golden outputs were computed from."""
    spec = C.ATTN_CASES[name]
    inp = C.attn_inputs(spec)
    z = _npz("attention_golden.npz")
    assert bytes(z[f"{name}/checksum"]).decode() == C.checksum(inp), f"input drift in {name}"
    gold = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(name + "/")}
    return spec, inp, gold


def gdn_case(name: str):
    spec = C.GDN_CASES[name]
    inp = C.gdn_inputs(spec)
    z = _npz("gdn_golden.npz")
    assert bytes(z[f"{name}/checksum"]).decode() == C.checksum(inp), f"input drift in {name}"
    gold = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(name + "/")}
    return spec, inp, gold


def module_case(name: str):
    spec = C.MODULE_CASES[name]
    w = C.module_weights(spec)
    inp = C.module_inputs(spec)
    z = _npz("module_golden.npz")
    assert bytes(z[f"{name}/checksum"]).decode() == C.checksum({**w, **inp}), f"input drift in {name}"
    gold = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(name + "/")}
    return spec, w, inp, gold


def prologue_case(name: str):
    spec = C.PROLOGUE_CASES[name]
    inp = C.prologue_inputs(spec)
    z = _npz("prologue_golden.npz")
    assert bytes(z[f"{name}/checksum"]).decode() == C.checksum(inp), f"input drift in {name}"
    gold = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(name + "/")}
    return spec, inp, gold


def state_pool_case(name: str):
    spec = C.STATE_POOL_CASES[name]
    inp = C.state_pool_inputs(spec)
    z = _npz("state_pool_golden.npz")
    assert bytes(z[f"{name}/checksum"]).decode() == C.checksum(inp), f"input drift in {name}"
    gold = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(name + "/")}
    return spec, inp, gold


def fp8_case(name: str):
    spec = C.FP8_CASES[name]
    inp = C.fp8_inputs(spec)
    z = _npz("fp8_golden.npz")
    assert bytes(z[f"{name}/checksum"]).decode() == C.checksum(inp), f"input drift in {name}"
    gold = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(name + "/")}
    return spec, inp, gold
