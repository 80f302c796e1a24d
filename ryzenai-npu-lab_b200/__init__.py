"""B200-native LFM2.5 decode attention (paged KV append + split-KV flash-decode).

Import with importlib (the directory name is not a Python identifier):

    pkg = importlib.import_module("ryzenai-npu-lab_b200")

Modules:
  _lib         ctypes binding of libb2attn.so (include/b2_decode_attn.h)
  build        nvcc build of libb2attn.so for sm_100a
  rope         host RoPE cos/sin tables (the reference computes them on the host)
  paged_cache  paged BF16 KV pool, block allocator, block tables
  attention    torch-facing wrappers and the PagedDecodeAttention runner
  operators    drop-in shims with the reference's NPU operator signatures
  distributed  sequence sharding and long-context split-KV across GPUs
  lfm2_runner  whole-token LFM2.5 decode runner (one CUDA graph per token)
  hf_paged     transformers adapter: "b200_paged" attention + B200PagedCache
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
