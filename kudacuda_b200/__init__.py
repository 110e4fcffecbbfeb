"""KudaCuda-B200: the NF4 batch-1 decode hot path of KudaCuda, rebuilt for
sm_100a behind the reference's C ABI and Python sidecar interface.

The compute lives in lib/libkudacuda.so (hand-written CUDA for sm_100a,
sources in csrc/); this package holds the ctypes bridge that mirrors the
reference's python/kudacuda_sidecar.py, the static CUDA-graph decode runner
and graph plan, and the Qwen2/Llama NF4 decode engine built on the C ABI.
"""

__all__ = ["native"]
