"""B200-native (sm_100a) routed-expert MoE hot path of slotstream-spark.

Layout:
* ``kernels/`` -- drop-in mirrors of the reference's ``slotstream_spark/kernels`` modules on this path
  (topk_stable, moe_align, moe_gemv_affine, fused_moe_affine, gemv_affine, gemm_affine) plus the additive
  fused entry points (router, moe_layer). Every launch goes through the C-ABI library ``libslotstream_b200.so``.
* ``records`` -- expert record byte layout for any (hidden, inter, gs).
* ``synth``   -- seeded synthetic workload (records, activations, router weights, Zipf bias).
"""
__version__ = "0.1.0"
