"""Record torch's CUDA bf16 sigmoid for the bf16 logits whose rounding depends on the
last bit of the fp32 ``exp`` (see ``oracle.dsalt_oracle.sigmoid_bf16``).

Runs on a CUDA machine (no reference code needed); writes
``tests/golden/sigmoid_bf16_cuda.npz`` (or the path given as argument): the bf16 bit
patterns of those logits and of their sigmoid, with the device and torch version.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import dsalt_oracle as O  # noqa: E402


def main():
    out = sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "sigmoid_bf16_cuda.npz")
    bits = np.arange(65536, dtype=np.uint32)
    vals = O.bf16_bits_to_f32(bits)
    fin = np.isfinite(vals)
    s_exact = O._sigmoid_exact(vals[fin])
    amb = O.sigmoid_ambiguous_f32(vals[fin], s_exact)
    cand = bits[fin][amb]
    x = torch.from_numpy(O.bf16_bits_to_f32(cand)).to(torch.bfloat16).cuda()
    s = torch.sigmoid(x).float().cpu().numpy()
    sig = np.array([int(O.f32_to_bf16_bits(v)) for v in s.tolist()], dtype=np.uint16)
    np.savez_compressed(out, logit_bits=cand.astype(np.uint16), sigmoid_bits=sig,
                        device=np.array(torch.cuda.get_device_name(0)), torch=np.array(torch.__version__))
    print(f"wrote {len(sig)} entries to {out}")


if __name__ == "__main__":
    main()
