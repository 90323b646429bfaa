"""Generates the golden fixtures in this folder by running the reference's own
behavioural model, legacy_100mhz_closed/src/PC/model_backend.py (and its RTL
rounding overlay, legacy_100mhz_closed/src/software/interactive/tests/
rtl_numeric_reference.py), on seeded synthetic assets written in the
reference's SD-card format by libqwen_b200's generator.

The reference checkout is only present where the fixtures are made; the GPU
machines only read the committed fixtures. Usage:

    python tests/golden/make_golden.py [--reference /path/to/reference]
"""
import argparse
import ctypes
import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / 'fpga2026-40999-llm-accelerator-for-qwen2.5-0.5b-on-fpga_b200'))

SEED = 2026
PROMPT_LEN = 16
STEPS = 6
DUMP_LAYERS = (0, 23)
ASSETS = ['CONFIG.JSON', 'DESC.BIN', 'SCALE.BIN', 'BIAS.BIN', 'GAMMA.BIN', 'WEIGHTS.BIN', 'LMW.BIN', 'EMBED.BIN']


def bf16_bits(t):
    """float32 torch tensor holding bf16 values -> uint16 bit patterns."""
    a = t.detach().float().contiguous().numpy()
    bits = a.view(np.uint32)
    assert not (bits & 0xffff).any(), 'tensor is not bf16-valued'
    return (bits >> 16).astype(np.uint16)


def step_record(logits, token):
    bits = bf16_bits(logits)
    vals = logits.numpy()
    order = np.lexsort((-np.arange(vals.size), -vals))[:8]  # value desc, then index desc
    return dict(token=int(token), top_ids=[int(i) for i in order], top_values=[float(vals[i]) for i in order],
                logits_sha256=hashlib.sha256(bits.tobytes()).hexdigest(), min=float(vals.min()),
                max=float(vals.max()))


def generate(model, prompt):
    ids, position, steps = list(prompt), 0, []
    logits0 = None
    for _ in range(STEPS):
        token = model.forward(ids, position)
        steps.append(step_record(model.last_logits, token))
        if logits0 is None:
            logits0 = bf16_bits(model.last_logits)
        position += len(ids)
        ids = [token]
    return steps, logits0


def teacher_forced(model, prompt):
    model.clear()
    out = []
    for i, tok in enumerate(prompt):
        nxt = model.forward([tok], i)
        out.append(step_record(model.last_logits, nxt))
    return out


def layer_dump(model, prompt):
    """Replays model_backend.Model.forward (:80-115) with the model's own
    operator methods to record the per-layer tensors of the prompt pass."""
    import torch
    m = model
    m.clear()
    rows = len(prompt)
    x = m.embedding[prompt]
    positions = torch.arange(0, rows).float()
    causal = torch.arange(rows)[None, :] > positions[:, None]
    dumps = {}
    with torch.inference_mode():
        for layer, weight in enumerate(m.weights):
            x_in = x.clone()
            h = m.norm(x, m.gamma[layer * 1792:layer * 1792 + 896])
            q = m.project_bias(h, weight['q'], m.bias[layer * 1152:layer * 1152 + 896]).reshape(rows, 14, 64)
            k = m.project_bias(h, weight['k'], m.bias[layer * 1152 + 896:layer * 1152 + 1024]).reshape(rows, 2, 64)
            v = m.project_bias(h, weight['v'], m.bias[layer * 1152 + 1024:layer * 1152 + 1152]).reshape(rows, 2, 64)
            q, k = m.rope(q, positions), m.rope(k, positions)
            keys, values = k.repeat_interleave(7, dim=1), v.repeat_interleave(7, dim=1)
            score = m.bf(torch.einsum('rhd,shd->hrs', q, keys) / 8.0)
            score.masked_fill_(causal[None, :, :], -float('inf'))
            probability = m.bf(torch.softmax(score, dim=-1))
            attn = m.bf(torch.einsum('hrs,shd->rhd', probability, values)).reshape(rows, 896)
            x = m.bf(x + m.linear(attn, weight['o']))
            hh = x.clone()
            z = m.norm(x, m.gamma[layer * 1792 + 896:(layer + 1) * 1792])
            gate, up = m.linear(z, weight['gate']), m.linear(z, weight['up'])
            mid = m.bf(m.bf(torch.nn.functional.silu(gate)) * up)
            x = m.bf(x + m.linear(mid, weight['down']))
            if layer in DUMP_LAYERS:
                for key, t in dict(x=x_in, q=q.reshape(rows, 896), k=k.reshape(rows, 128), v=v.reshape(rows, 128),
                                   context=attn, h=hh, m=mid, y=x).items():
                    dumps[f'layer{layer}_{key}'] = bf16_bits(t)
        logits = m.linear(m.norm(x[-1:], m.gamma[43008:]), m.lm).flatten()
        token = logits.numel() - 1 - int(torch.argmax(logits.flip(0)))
    return dumps, token


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', type=Path, default=Path('/root/reference'))
    ap.add_argument('--threads', type=int, default=8)
    args = ap.parse_args()
    sys.path.insert(0, str(args.reference / 'legacy_100mhz_closed/src/PC'))
    sys.path.insert(0, str(args.reference / 'legacy_100mhz_closed/src/software/interactive/tests'))
    import torch
    from model_backend import Model
    from rtl_numeric_reference import configure_reference

    import qwen_b200
    L = qwen_b200.lib()
    prompt_arr = (ctypes.c_uint32 * PROMPT_LEN)()
    L.qwen_b200_synth_prompt(SEED, PROMPT_LEN, prompt_arr)
    prompt = [int(v) for v in prompt_arr]
    with tempfile.TemporaryDirectory() as tmp:
        assert L.qwen_b200_synth_write(tmp.encode(), SEED) == 0
        hashes = {name: hashlib.sha256((Path(tmp) / 'QWEN25' / name).read_bytes()).hexdigest() for name in ASSETS}
        model = Model(tmp, threads=args.threads)
        steps, logits0 = generate(model, prompt)
        forced = teacher_forced(model, prompt)
        dumps, dump_token = layer_dump(model, prompt)
        assert dump_token == steps[0]['token'], 'replayed forward disagrees with Model.forward'
        rtl = configure_reference(Model(tmp, threads=args.threads))
        rtl_steps, rtl_logits0 = generate(rtl, prompt)
    golden = dict(
        seed=SEED, prompt=prompt, asset_sha256=hashes,
        generator='libqwen_b200 qwen_b200_synth_write (fp32 N(0,0.02) -> int8 per output channel)',
        reference='legacy_100mhz_closed/src/PC/model_backend.py (torch %s, CPU)' % torch.__version__,
        generate=steps, teacher_forced=forced, rtl_boundaries_generate=rtl_steps,
        dump_layers=list(DUMP_LAYERS))
    (HERE / f'qwen_seed{SEED}.json').write_text(json.dumps(golden, indent=1) + '\n')
    np.savez_compressed(HERE / f'qwen_seed{SEED}.npz', logits_step0=logits0, rtl_logits_step0=rtl_logits0, **dumps)
    print(json.dumps(dict(tokens=[s['token'] for s in steps], forced=[s['token'] for s in forced],
                          rtl=[s['token'] for s in rtl_steps])))


if __name__ == '__main__':
    main()
