"""CPU oracle for the gpt-oss MXFP4 MoE path: test infrastructure, not product.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference-arm legs may import it. The CUDA
library in gptoss-infer_b200/ never routes through it: there is no CPU fallback.
"""
