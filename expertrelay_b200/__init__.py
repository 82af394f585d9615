"""expertrelay_b200: ExpertRelay's MoE-block hot path on B200 (sm_100a).

  expertrelay_b200.moe.MoeBlock         one MoE layer in HBM, run by er_moe_block
  expertrelay_b200.backend.B200Backend  the reference's compute-backend protocol
  expertrelay_b200.store                expert record layouts (store/layout.py, store/int4.py)
  expertrelay_b200.quant                store weight encodings (int8, int4, GPTQ v1)
  expertrelay_b200.synth                seeded synthetic blocks and activations
  expertrelay_b200.build                nvcc build of libexpertrelay_b200.so
"""

__version__ = "0.1.0"
