"""mdlc_b200 — B200-native (sm_100a) execution backend for mdlc's Graph IR.

``mdlc_b200.compile(graph)`` takes the reference compiler's passes-optimised
Graph IR and returns an :class:`~mdlc_b200.compiler.Executable` that runs it
through the prebuilt ``libmdlc_b200.so`` (tcgen05 implicit-GEMM convolution,
memory-bound depthwise / pooling / elementwise kernels).
"""

__version__ = "0.1.0"


def compile(graph, **kwargs):
    """See :func:`mdlc_b200.compiler.compile`."""
    from mdlc_b200.compiler import compile as _compile
    return _compile(graph, **kwargs)
