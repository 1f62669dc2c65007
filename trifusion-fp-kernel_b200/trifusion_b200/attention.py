"""FP32 masked attention (reference ``attention.py:8-18``).

Projections stay BF16; the attention itself runs in FP32 through PyTorch's
scaled-dot-product attention (memory-efficient or math backend), as the
reference validates it, and returns the input dtype.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel


def masked_attention(q, k, v, mask, out_dtype=None):
    """``out_dtype`` defaults to q's dtype; FP32 operands may be given directly
    (the B200 rotary kernel writes them) with a BF16 result requested."""
    out_dtype = q.dtype if out_dtype is None else out_dtype
    with torch.autocast(q.device.type, enabled=False), sdpa_kernel(
            [SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]):
        if out_dtype in (torch.float16, torch.bfloat16):
            q, k, v = q.float(), k.float(), v.float()
        return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, dropout_p=0.0).to(out_dtype)
