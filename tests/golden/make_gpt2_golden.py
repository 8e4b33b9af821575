"""Generates the GPT-2 124M greedy-decode fixture from the CPU oracle.

Workload: GptModel::load_random(GptConfig{50257, 768, 12, 12, 3072, 1024,
1e-5}, seed 3) (crates/open-cuda-llm/src/lib.rs:635-646), the fused flash
attention path (block 64, llm:374-387 with blas:589-678), greedy generate
of 128 new tokens (llm:910-929) from each of the 32 prompts of
synth.gpt_prompts(32, 32) (32 ids from SplitMix64(3 + 1000*(b+1)) mod the
vocabulary).  Sequence 0 is also the batch-1 workload.

Stored (tests/golden/gpt2_124m_seed3_128tok.npz, ~0.5 MB):
  prompts [32][32] u32, tokens [32][128] u32,
  top2 [32][128] u32 (the runner-up id at every step) and margin
  [32][128] f32 (top-1 minus top-2 logit), for diagnosing a mismatch,
  sub_idx [256] u32: fixed vocabulary ids; sub_seq0 [128][256] f32: the
  logits of sequence 0 at those ids for every step; sub_last [32][256] f32:
  every sequence's last-step logits at those ids,
  full_seq0_last [50257] f32: sequence 0's full last-step logits.

    python tests/golden/make_gpt2_golden.py        (about 5 minutes, all cores)
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    sys.path.insert(0, p)

import oracle  # noqa: E402
import synth  # noqa: E402

OUT = os.path.join(HERE, "gpt2_124m_seed3_128tok.npz")
BATCH, PROMPT, NEW, SEED, BLOCK, NSUB = 32, 32, 128, 3, 64, 256


def main():
    cfg = oracle.GptConfig.gpt2_124m()
    model = oracle.GptModel(cfg, SEED)
    model.set_attention(flash=True, block=BLOCK)
    prompts = synth.gpt_prompts(BATCH, PROMPT)
    sub_idx = (synth.splitmix64(77, NSUB) % np.uint64(cfg.vocab_size)).astype(np.uint32)
    tokens = np.zeros((BATCH, NEW), np.uint32)
    top2 = np.zeros((BATCH, NEW), np.uint32)
    margin = np.zeros((BATCH, NEW), np.float32)
    sub_last = np.zeros((BATCH, NSUB), np.float32)
    t0 = time.time()
    for b in range(BATCH):
        toks, lg = model.generate(prompts[b], NEW, want_logits=True)
        assert len(toks) == NEW
        tokens[b] = toks
        order = np.argsort(-lg, axis=1, kind="stable")[:, :2]
        top2[b] = order[:, 1]
        margin[b] = lg[np.arange(NEW), order[:, 0]] - lg[np.arange(NEW), order[:, 1]]
        sub_last[b] = lg[-1, sub_idx]
        if b == 0:
            sub_seq0 = lg[:, sub_idx].copy()
            full_seq0_last = lg[-1].copy()
        print(f"sequence {b}: {time.time() - t0:.1f} s", flush=True)
    np.savez_compressed(OUT, prompts=prompts, tokens=tokens, top2=top2, margin=margin, sub_idx=sub_idx,
                        sub_seq0=sub_seq0, sub_last=sub_last, full_seq0_last=full_seq0_last, seed=SEED,
                        block=BLOCK)
    print("wrote", OUT)


if __name__ == "__main__":
    main()
