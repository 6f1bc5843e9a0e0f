"""Drop-in for ``longcat_kernel.longcat_flash_attn``.

Reference: hy-worldplay/files/hyvideo/models/transformers/modules/longcat_kernel.py:158-233
and matrix-game-3.0/files/wan/modules/longcat_kernel.py:137-190. The Triton
kernel ``_attn_fwd_bsa_align`` is replaced by the sm_100a tcgen05 kernel behind
``li_sparse_attn_tiled``.

Same arguments, same errors (``ValueError`` for a key length that is not a
block multiple or an index past the last key block). Two deliberate
differences:

* query rows are grouped by ``logical_block_size``: query block ``i`` uses
  index row ``i``. The reference fixes ``BLOCK_M = 128``, so with 64-token
  blocks its query block ``2m+1`` reuses row ``m``'s list; this backend applies
  every row's own list.
* inputs that are not fp16/bf16 are cast to bf16 for the attention (as the
  Matrix-Game copy does, ``:139-147``) and the output is returned in q's dtype.
"""

from __future__ import annotations

import torch

from . import kernels as K


def longcat_flash_attn(q, k, v, block_indices, block_counts, sm_scale=None, logical_block_size=128,
                       validate=True):
    """Block-sparse flash attention over tiled ``[B, H, L, D]`` tensors.

    ``validate=False`` skips the host-side index bound check (which, as in the
    reference, reads ``block_indices.max()`` and so synchronises); the kernel
    still guards every index on the device, but asynchronously: an out-of-range
    block id is read as block 0 and sets ``LI_DEVERR_BAD_INDEX`` in the device
    error word, and this call returns normally. ``kernels.raise_device_errors()``
    (a synchronising read, e.g. at a step boundary) turns that into the
    reference's ``ValueError``.
    """
    B, H, Q_len, D = q.shape
    K_len = k.shape[2]
    if sm_scale is None:
        sm_scale = 1.0 / (D ** 0.5)
    BLOCK_N = logical_block_size
    if K_len % BLOCK_N != 0:
        raise ValueError(f"K Length ({K_len}) must be divisible by logical_block_size ({BLOCK_N})")
    block_indices = block_indices.to(torch.int32)
    block_counts = block_counts.to(torch.int32)
    if validate and block_indices.numel() and int(block_indices.max()) >= (K_len // BLOCK_N):
        raise ValueError("Sparse indices out of bounds.")
    return K.sparse_attn_tiled(q, k, v, block_indices, block_counts, BLOCK_N, sm_scale)
