"""Generate the golden fixture of the attention backward by differentiating the reference's
PyTorch restatement of its kernel on CPU.

Run in a container where the reference is mounted (it is never read at test time):

    PYTHONPATH=/path/to/dsalt TORCHDYNAMO_DISABLE=1 python tests/golden/make_golden_backward.py

``_block_attention`` (``results/causal_landmark_check.py:119-147``: window keys
``[i−w(i)+1, i]`` plus the landmarks ``p ≤ i``, ``p < i−w(i)+1`` of the query block's set,
softmax in fp32) is run on seeded q, k, v for every 256-query block of one sequence, each
block with its own landmark set, and differentiated by autograd for a seeded output
gradient: the gradients of q, k and v that the reference's Triton backward
(``dsalt/kernels/dsalt_triton_bwd.py``) computes. Output: ``bwd_ref.npz``.
"""
from __future__ import annotations

import math
import os

import numpy as np
import torch

from results.causal_landmark_check import _block_attention

HERE = os.path.dirname(os.path.abspath(__file__))
L, H, D, K, BLOCK, SEED = 512, 2, 8, 12, 256, 21


def main():
    g = torch.Generator().manual_seed(SEED)
    q = torch.randn(L, H, D, generator=g).requires_grad_(True)
    k = torch.randn(L, H, D, generator=g).requires_grad_(True)
    v = torch.randn(L, H, D, generator=g).requires_grad_(True)
    w = torch.randint(1, 200, (L,), generator=g, dtype=torch.int32)
    n_sets = L // BLOCK
    lmk = torch.empty(H, n_sets, K, dtype=torch.int64)
    for b in range(n_sets):
        for h in range(H):
            lmk[h, b] = torch.randperm((b + 1) * BLOCK, generator=g)[:K]
    lmk[0, 1, -2:] = -1  # empty slots
    scale = 1.0 / math.sqrt(D)
    out = torch.cat([_block_attention(q, k, v, w, lmk[:, b], b * BLOCK, (b + 1) * BLOCK, scale)
                     for b in range(n_sets)], 0)
    dout = torch.randn(L, H, D, generator=g)
    (out * dout).sum().backward()
    np.savez_compressed(os.path.join(HERE, "bwd_ref.npz"), q=q.detach().numpy(), k=k.detach().numpy(),
                        v=v.detach().numpy(), w=w.numpy(), lmk=lmk.to(torch.int32).numpy(), block=BLOCK,
                        out=out.detach().numpy(), dout=dout.numpy(), dq=q.grad.numpy(), dk=k.grad.numpy(),
                        dv=v.grad.numpy())


if __name__ == "__main__":
    main()
