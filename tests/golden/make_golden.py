"""Generates the greedy-decode golden fixtures with the CPU oracle.

Run from the repository root:  python tests/golden/make_golden.py
Writes tests/golden/decoder_greedy.json: for each case the synthetic model
(seeded, aiimage_b200.synth), the prompt seed and length, the 64 greedy token
ids, the top-1/top-2 logit margin at every step (a near-tie would make a
token flip a numerics question rather than a bug) and the 20 largest logits
of the last step.
"""
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as O  # noqa: E402
from aiimage_b200 import synth  # noqa: E402

CASES = {
    # 24-layer Q4 g32 decoder, 512-token prompt, 64 greedy tokens.
    "qwen35_08b_q4_prompt512": dict(cfg="QWEN35_08B_Q4", seed=3, prompt_len=512, prompt_seed=30, max_new=64),
    # The Q8 per-row variant of the same model (config 4's weights), shorter prompt.
    "qwen35_08b_q8_prompt64": dict(cfg="QWEN35_08B_Q8", seed=4, prompt_len=64, prompt_seed=40, max_new=64),
}


def run(case):
    cfg = getattr(synth, case["cfg"])
    model = synth.SyntheticDecoder(cfg, seed=case["seed"])
    prompt = model.prompt(case["prompt_len"], seed=case["prompt_seed"])
    dec = O.OracleDecoder(model)
    t = time.time()
    toks, margins = dec.generate(prompt, case["max_new"])
    top = sorted(range(len(dec.last_logits)), key=lambda i: (-dec.last_logits[i], i))[:20]
    return dict(case, tokens=toks, margins=[float(m) for m in margins], oracle_seconds=round(time.time() - t, 1),
                oracle_threads=O.num_threads(), last_top20_ids=top,
                last_top20_logits=[float(dec.last_logits[i]) for i in top])


if __name__ == "__main__":
    O.build()
    out = {name: run(c) for name, c in CASES.items()}
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "decoder_greedy.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    for name, c in out.items():
        print(name, c["tokens"][:8], "min margin", min(c["margins"]), c["oracle_seconds"], "s")
