"""Record the state-dict layout (key -> shape) of the reference's decoder
(``dsalt/model/dsalt_lm.py:64`` ``DSALTLMHeadModel``) for the small configuration of
``tests/test_model.py``, so that the test checks the layout without the reference present.

Run in a container where the reference is mounted:

    PYTHONPATH=/path/to/dsalt python tests/golden/make_lm_keys.py
"""
import json
import os

from dsalt.model.dsalt_lm import DSALTLMHeadModel

HERE = os.path.dirname(os.path.abspath(__file__))
SMALL = dict(vocab_size=1000, d_model=256, n_layers=2, n_heads=4, n_min=16, n_max=128, k_lmk=32, max_seq_len=4096)

if __name__ == "__main__":
    ref = DSALTLMHeadModel(**SMALL, n_kv_heads=2, qkv_bias=True)
    layout = {k: list(v.shape) for k, v in ref.state_dict().items()}
    with open(os.path.join(HERE, "lm_state_dict_small.json"), "w") as f:
        json.dump({"config": dict(SMALL, n_kv_heads=2, qkv_bias=True), "state_dict": layout}, f, indent=0,
                  sort_keys=True)
