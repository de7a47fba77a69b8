"""Writes the golden fixtures of tests/golden from the CPU oracle (oracle/), run on small seeded
cases of the benchmark configurations.

The reference is Go and cannot run on these machines, and its tests hold no numeric golden
vectors of this path (internal/golden/testdata holds SHA-256 hashes that need Go's math/rand and a
training run). The oracle is pinned instead by the reference tests' own known answers
(reference_kats.json, checked in test_golden.py) and properties (test_oracle_*.py); these
fixtures freeze its outputs so that the CUDA path is checked against committed numbers, on a GPU
box that has neither the reference nor a rebuilt oracle.

    python tests/golden/make_golden.py      # rewrites tests/golden/*.npz
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from mignon_ai_b200 import synth  # noqa: E402
import pyoracle  # noqa: E402

# (name, config, vocab, sessions, prompt length, greedy steps, prompt seed)
GENERATE = [
    ("config1", 1, 1024, 8, 32, 8, 1),
    ("config2", 2, 512, 8, 48, 8, 2),
]
SCORE = ("config4", 4, 512, 4, 64, 4)  # name, config, vocab, sequences, length, seed
POLICY = ("policy", 2, 512, 6, 24, 8, 7)  # name, config, vocab, sessions, prompt, steps, seed


def spec_of(cfg, vocab):
    return synth.ModelSpec(**{**synth.CONFIGS[cfg].__dict__, "vocab": vocab})


def main():
    pyoracle.lib()
    for name, cfg, vocab, n, P, steps, seed in GENERATE:
        om = pyoracle.Model(synth.build_model_file(spec_of(cfg, vocab)))
        prompts = synth.prompts_uniform_fast(n, P, vocab, seed=seed)
        lens = np.full(n, P, np.int32)
        lens[1], lens[n - 1] = P // 2, 1
        toks, probs, logits = om.generate_greedy(prompts, lens, steps, logits=True)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), config=cfg, vocab=vocab, prompts=prompts, lens=lens,
                            tokens=toks, probs=probs, logits=logits)
    name, cfg, vocab, n, L, seed = SCORE
    om = pyoracle.Model(synth.build_model_file(spec_of(cfg, vocab)))
    seqs = synth.prompts_uniform_fast(n, L, vocab, seed=seed)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), config=cfg, vocab=vocab, seqs=seqs, logprobs=om.score(seqs))
    name, cfg, vocab, n, P, steps, seed = POLICY
    om = pyoracle.Model(synth.build_model_file(spec_of(cfg, vocab)))
    prompts = synth.prompts_uniform_fast(n, P, vocab, seed=seed)
    lens = np.full(n, P, np.int32)
    sp = pyoracle.Sampling(0.7, 1.2, 40, 0.9, 6, 1)
    toks, probs, out_lens, logits = om.generate_policy(prompts, lens, steps, sp, penalize_prompt=True, session0=seed,
                                                       logits=True)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), config=cfg, vocab=vocab, prompts=prompts, lens=lens,
                        session0=seed, sampling=np.array([0.7, 1.2, 40, 0.9, 6, 1], np.float64), tokens=toks,
                        probs=probs, out_lens=out_lens, logits=logits)


if __name__ == "__main__":
    main()
