"""Drop-in backend modules for ``gemm_compare.backends``: ``nvfp`` and ``mxfp`` keep the reference's
state classes, (de)serialisers and ``build_*_fns`` builders (gemm_compare/backends/nvfp.py,
mxfp.py), with ``quant_fn`` and ``emul_fn`` running on libemugen.so and ``real_fn`` on the hardware FP4
GEMM from flashinfer.  The reference's own factory (gemm_compare/backends/__init__.py:20-42) selects
between the two modules by name and needs nothing from this package.
"""
