"""Continuous batching on the B200: more requests than sequence slots, prompts
split over several steps by a small prefill budget, requests joining and
leaving the batch at different steps. Every request's tokens must equal
greedy generation of that request alone (qwen_b200_forward, the
model_backend.py:80-115 interface), with the reference loop's stop ids
(151643 / 151645, src/software/generation.c)."""
import numpy as np
import pytest

import qwen_b200

pytestmark = pytest.mark.gpu
EOS = (151643, 151645)


def alone(engine, prompt, max_new):
    engine.reset(0)
    tok, _ = engine.forward(0, prompt, 0)
    out, pos = [tok], len(prompt)
    while len(out) < max_new and out[-1] not in EOS:
        tok, _ = engine.forward(0, [out[-1]], pos)
        pos += 1
        out.append(tok)
    return out


def test_scheduler_matches_requests_run_alone(sd_root):
    e = qwen_b200.Engine(device=0, max_seqs=3, max_context=256, max_rows=64).load_assets(sd_root)
    try:
        r = np.random.default_rng(8)
        lens, news = [40, 7, 90, 23, 64, 5], [6, 3, 8, 1, 5, 4]
        prompts = [r.integers(0, 151936, n).astype(np.uint32) for n in lens]
        s = qwen_b200.Scheduler(e, prefill_budget=50)
        rids = [s.submit(p, m) for p, m in zip(prompts, news)]
        steps = 0
        while s.step():
            steps += 1
            assert steps < 200
        got = {}
        for rid in rids:
            toks, done = s.result(rid)
            assert done
            got[rid] = toks
        s.close()
        for rid, p, m in zip(rids, prompts, news):
            assert got[rid] == alone(e, p, m), rid
    finally:
        e.close()
