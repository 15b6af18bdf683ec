"""stealcode_b200 -- B200 (sm_100a) implementation of the streaming
Nemotron/FastConformer encoder hot path of she-workss/stealcode.

The product is ``libstealcode_cuda.so`` (C ABI: ``include/stealcode_b200.h``);
this package holds its CUDA sources (``csrc/``), the build step (``build``),
the ctypes binding (``_lib``), a host-side mirror of the reference operator
interface (``ops``) and the seeded synthetic-input generator (``synth``).

Operator names are resolved lazily so that ``python -m stealcode_b200.build``
works before the library exists; any use of an operator imports ``_lib``,
which raises ImportError when the library is missing (there is no fallback).
"""
_OPS = {"AttnStreamKernel", "Lin", "Q8Mat", "StreamEncoder", "attn_stream_ring", "q8_gemm", "quantize"}


def __getattr__(name):
    if name in _OPS:
        from . import ops

        return getattr(ops, name)
    raise AttributeError(name)
