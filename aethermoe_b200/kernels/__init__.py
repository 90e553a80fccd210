"""Drop-in modules with the reference's kernel API (``src/kernels/*.py``).

Put this directory on ``sys.path`` (as the reference's tests do with its own
``src/kernels``) and ``from fused_gating_metal import fused_gating`` resolves
to the B200 implementation.  Each function keeps the reference's name,
argument order, output layout and error behaviour; the compute runs in
``libaethermoe.so`` on the GPU.
"""
