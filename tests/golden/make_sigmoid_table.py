"""Record torch's CUDA bf16 sigmoid for the bf16 logits whose rounding depends on the
last bit of the fp32 ``exp`` (see ``oracle.dsalt_oracle.sigmoid_bf16``).

Runs on a CUDA machine (no reference code needed); writes
``tests/golden/sigmoid_bf16_cuda.json`` (or the path given as argument).
"""
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import dsalt_oracle as O  # noqa: E402


def main():
    out = sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "sigmoid_bf16_cuda.json")
    bits = np.arange(65536, dtype=np.uint32)
    vals = O.bf16_bits_to_f32(bits)
    fin = np.isfinite(vals)
    s_exact = O._sigmoid_exact(vals[fin])
    amb = O.sigmoid_ambiguous_f32(vals[fin], s_exact)
    cand = bits[fin][amb]
    x = torch.from_numpy(O.bf16_bits_to_f32(cand)).to(torch.bfloat16).cuda()
    s = torch.sigmoid(x).float().cpu().numpy()
    table = {int(b): int(O.f32_to_bf16_bits(v)) for b, v in zip(cand.tolist(), s.tolist())}
    with open(out, "w") as fh:
        json.dump({"device": torch.cuda.get_device_name(0), "torch": torch.__version__,
                   "cuda_sigmoid_bf16_bits": table}, fh, indent=1)
    print(f"wrote {len(table)} entries to {out}")


if __name__ == "__main__":
    main()
