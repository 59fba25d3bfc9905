"""B200 (sm_100a) cascade-decode operator set.

``import cascade_kernel`` loads the native extension and registers, for CUDA
tensors, the reference's torch ops (``torch.ops.npu.fa_fp32_stage1``,
``torch.ops.npu.lse_merge``, ``torch.ops.npu.f3_gateup_epilogue``) plus the
extended-domain siblings (``cascade_prefix_attention``,
``cascade_suffix_decode``, ``cascade_lse_merge``, ``cascade_gateup_swiglu``).
Like the reference package (ascend-kernel/python/ascend_kernel/ascend_kernel/
__init__.py:5-15) it only loads the library; it never imports vllm.

There is no fallback: if the native library is missing the import fails.
"""
import os

import torch

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib")
_EXT = os.path.join(LIB_DIR, "_C.so")
CAPI_PATH = os.path.join(LIB_DIR, "libcascade_b200.so")

if not os.path.exists(_EXT):
    raise ImportError(
        "cascade_kernel: native extension not built (run "
        "`python vllm-hust-cascade-kernel_b200/build.py`); there is no CPU fallback")
torch.ops.load_library(_EXT)

from . import cascade  # noqa: E402,F401  composed cascade step helpers

__all__ = ["LIB_DIR", "CAPI_PATH", "cascade"]
