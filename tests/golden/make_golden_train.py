"""Generate the golden fixture of the soft-selector training attention by running the
reference (LeonardoCofone/dsalt) on CPU.

Run in a container where the reference is mounted (it is never read at test time):

    PYTHONPATH=/path/to/dsalt TORCHDYNAMO_DISABLE=1 python tests/golden/make_golden_train.py

For each case below, with a seeded ``DSALTAttention`` in training mode and seeded inputs, it
records from the reference's own functions:

* ``_train_selectors`` (``dsalt/modules/dsalt_attention.py:457-487``): the continuous widths
  ``w_cont``, the landmark positions ``lmk_pos`` and their log-weights ``lmk_logw``, and the
  hybrid scores ``hybrid_scores_per_head`` (``dsalt/kernels/landmark_tokens_ker.py:19-61``)
  they are taken from;
* the dense training attention of ``_packed_train`` (``dsalt_attention.py:489-515``): the
  log-bias ``_dense_logbias_from_kernel`` (``:517-563``, the math of the Triton training
  kernel) and ``scaled_dot_product_attention``, on seeded q, k, v (grouped kv heads repeated
  as ``_repeat_kv`` does), its output and, for a seeded output gradient, the autograd
  gradients of q, k, v (per kv head), ``w_cont`` and ``lmk_logw``.

Everything runs in fp32, as the reference's CPU path does. Output: ``train_ref.npz``, the
arrays of case ``c`` under keys ``c/<name>``.
"""
from __future__ import annotations

import os

import numpy as np
import torch
import torch.nn.functional as F

from dsalt.modules.dsalt_attention import DSALTAttention

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [
    dict(name="mha", seed=11, d_model=64, H=2, Hkv=2, n_min=4, n_max=40, k=6, N=2, L=64),
    dict(name="gqa", seed=12, d_model=64, H=4, Hkv=2, n_min=3, n_max=48, k=8, N=2, L=80),
]


def run_case(c):
    torch.manual_seed(c["seed"])
    H, Hkv, N, L = c["H"], c["Hkv"], c["N"], c["L"]
    D = c["d_model"] // H
    T = N * L
    m = DSALTAttention(c["d_model"], H, c["n_min"], c["n_max"], c["k"], max_seq_len=L, n_kv_heads=Hkv)
    m.train()
    with torch.no_grad():
        m.win_gate.weight.mul_(4.0)  # widths spread over [n_min, n_max]
    x = torch.randn(T, c["d_model"])
    cu_list = [s * L for s in range(N + 1)]
    cu = torch.tensor(cu_list, dtype=torch.int32)
    with torch.no_grad():
        w_cont, lmk_pos, lmk_logw = m._train_selectors(x, cu, T, x.device, cu_list)
        from dsalt.kernels.landmark_tokens_ker import hybrid_scores_per_head
        scores, _, _ = hybrid_scores_per_head(x, m.v_proj.weight, m._alpha(), H, D)
    g = torch.Generator().manual_seed(c["seed"] + 100)
    q = torch.randn(T, H, D, generator=g).requires_grad_(True)
    kg = torch.randn(T, Hkv, D, generator=g).requires_grad_(True)
    vg = torch.randn(T, Hkv, D, generator=g).requires_grad_(True)
    wl = w_cont.detach().clone().requires_grad_(True)
    ll = lmk_logw.detach().clone().requires_grad_(True)
    k, v = m._repeat_kv(kg), m._repeat_kv(vg)
    logbias = m._dense_logbias_from_kernel(wl, lmk_pos, ll, N, L, x.device)  # [N, H, L, L]
    qb, kb, vb = (t.view(N, L, H, D).transpose(1, 2) for t in (q, k, v))
    ob = F.scaled_dot_product_attention(qb, kb, vb, attn_mask=logbias.to(qb.dtype))
    out = ob.transpose(1, 2).reshape(T, H, D)
    dout = torch.randn(T, H, D, generator=g)
    (out * dout).sum().backward()
    arrays = dict(
        x=x, v_proj_weight=m.v_proj.weight.detach(), alpha=m._alpha().detach(), scores=scores, cu=cu,
        w_cont=w_cont, lmk_pos=lmk_pos.to(torch.int32), lmk_logw=lmk_logw, q=q.detach(), k=kg.detach(),
        v=vg.detach(), out=out.detach(), dout=dout, dq=q.grad, dk=kg.grad, dv=vg.grad, d_w=wl.grad, d_logw=ll.grad,
        tau=torch.tensor(m.tau_win), edge=torch.tensor(float(m.win_edge)), tau_lmk=torch.tensor(m.tau_lmk),
    )
    return {f"{c['name']}/{k_}": v_.detach().numpy() for k_, v_ in arrays.items()}


def main():
    torch.set_num_threads(4)
    out = {}
    for c in CASES:
        out.update(run_case(c))
        print(c["name"], "done")
    np.savez_compressed(os.path.join(HERE, "train_ref.npz"), **out)


if __name__ == "__main__":
    main()
