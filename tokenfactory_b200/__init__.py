"""tokenfactory_b200 - B200-native (sm_100a) hot path of tokenFactory's hybrid attention.

Drop-in for the data-parallel hot path of yz29528/tokenFactory's Qwen3.8 hybrid model:
  * paged GQA full attention (qwen3_8/full_attention.py): KV-pool store, decode and varlen extend
    over a radix-cached prefix through req_to_token, output gate;
  * Gated DeltaNet linear attention (qwen3_8/linear_attention.py): causal conv1d with rolling
    conv state, recurrent decode, varlen extend, gated RMSNorm epilogue.

Layers:
  include/tfattn.h + csrc/  - CUDA kernels behind a C ABI (libtfattn.so, built in-tree)
  _capi                     - ctypes binding of that ABI
  ops                       - torch-tensor entry points (one per C entry point)
  hybrid_attention          - the reference's method surface (_slot_based_attention,
                              _batched_decode_step, ...) re-expressed on the kernels, and the
                              mixins that install them into the reference's module classes
  forward_batch             - ForwardBatch with the reference's fields
"""

from .forward_batch import ForwardBatch  # noqa: F401

__all__ = ["ops", "ForwardBatch"]


def __getattr__(name):
    # ops loads the compiled extension; it is imported on first use, so that the package (and
    # its build module, `python -m tokenfactory_b200.build`) imports before anything is built
    if name == "ops":
        import importlib
        return importlib.import_module(__name__ + ".ops")
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
