#!/usr/bin/env python
"""Decode throughput of libqwen_b200 on B200s (one process per GPU).

Workload (a "step"): one greedy decode step of the seeded random-int8
Qwen2.5-0.5B for 64 independent sequences per GPU, each at context 2048+
(batched decode serving; the KV8 caches are filled with seeded synthetic codes
so the long prefill is not part of the measurement). Request-sharded: every
rank holds a full replica and its own 64 sequences, no data-path collective
(weak scaling). value = all ranks' tokens / max-over-ranks device time.

Also reported: e2e (the same step through the host-buffer C ABI call
qwen_b200_decode_step, H2D ids and D2H tokens inside the timed region), bs1
decode at short context (16-token prompt, the reference's CPU-runnable case),
per-kernel-class device times from CUDA events, the roofline of the dominant
kernel class and of the whole step, clocks sampled during the timed region,
and the oracle (CPU port of the reference model) timed on the host cores.

    python bench.py [--gpus N] [--steps K] [--warmup W]
    python bench.py --impl reference ...   # the CPU reference path alone
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
PKG = REPO / 'fpga2026-40999-llm-accelerator-for-qwen2.5-0.5b-on-fpga_b200'
for _p in (str(PKG), str(REPO)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

SEED = 2026
HID, FFN, QKV, VOCAB, LAYERS = 896, 4864, 1152, 151936, 24
KV_BYTES_PER_TOKEN_LAYER = 2 * 2 * (64 + 4)  # K and V, 2 heads, 64 codes + fp32 scale
CLASSES = ['embedding', 'qkv_rope_kv8', 'attention', 'o_proj_residual', 'gate_up_swiglu', 'down_residual',
           'lm_head_argmax', 'bookkeeping', 'persistent_decode']
# kernels behind each class: one row runs the GEMV family, more rows the
# tcgen05 GEMM (qkv/o/gate_up/down/LM head); attention is one launch of the
# register-layout kernel (every workload here)
KERNEL_NAMES_GEMV = {'qkv_rope_kv8': 'qkv_kernel', 'attention': 'attn_rs_kernel',
                     'o_proj_residual': 'gemv_kernel<896,EPI_RESIDUAL>',
                     'gate_up_swiglu': 'gemv_kernel<896,EPI_SWIGLU>',
                     'down_residual': 'gemv_kernel<4864,EPI_RESIDUAL>',
                     'lm_head_argmax': 'lm_head1_kernel + argmax_reduce_kernel',
                     'embedding': 'embed_kernel', 'bookkeeping': 'decode_prologue/epilogue_kernel',
                     'persistent_decode': 'decode1_kernel'}
KERNEL_NAMES_TC = dict(KERNEL_NAMES_GEMV,
                       qkv_rope_kv8='rmsnorm_limbs_kernel + tc_gemm_kernel<EPI_BIAS> + rope_kv8_kernel',
                       o_proj_residual='act_quant_kernel<896> + tc_gemm_kernel<EPI_RESIDUAL>',
                       gate_up_swiglu='rmsnorm_limbs_kernel + tc_gemm_kernel<EPI_SWIGLU>',
                       down_residual='act_quant_kernel<4864> + tc_gemm_kernel<EPI_RESIDUAL>',
                       lm_head_argmax='rmsnorm_limbs_kernel + tc_lmhead_kernel + argmax_reduce_kernel')


def kernel_names(rows):
    return KERNEL_NAMES_TC if rows > 1 else KERNEL_NAMES_GEMV


def weight_bytes():
    """Algorithmic bytes that one decode step reads once, whatever the batch."""
    layer = (QKV * HID + HID * HID + 2 * FFN * HID + HID * FFN  # int8 codes
             + 4 * (QKV + HID + 2 * FFN + HID)                   # fp32 scales
             + 2 * QKV + 2 * 2 * HID)                            # bf16 bias, gains
    return LAYERS * layer + VOCAB * HID + 4 * VOCAB + 2 * HID


def class_bytes(n, contexts):
    """Algorithmic bytes per launch of each kernel class for a step of n rows."""
    kv = sum(contexts) * KV_BYTES_PER_TOKEN_LAYER
    return {
        'embedding': n * HID * 2 * 2,
        'qkv_rope_kv8': QKV * HID + 4 * QKV + 2 * QKV + 2 * HID + n * HID * 2 * 2 + n * 2 * 2 * (64 + 4),
        'attention': kv + n * HID * 2 * 2,
        'o_proj_residual': HID * HID + 4 * HID + n * HID * 2 * 3,
        'gate_up_swiglu': 2 * FFN * HID + 4 * 2 * FFN + 2 * HID + n * HID * 2 + n * FFN * 2,
        'down_residual': HID * FFN + 4 * HID + n * FFN * 2 + n * HID * 2 * 2,
        'lm_head_argmax': VOCAB * HID + 4 * VOCAB + 2 * HID + n * HID * 2 + n * 4,
        'bookkeeping': n * 16,
    }


def step_bytes(contexts):
    return weight_bytes() + sum(contexts) * KV_BYTES_PER_TOKEN_LAYER * LAYERS


def peaks():
    p = REPO / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return float(d['hbm_gbs']), 'measured'
    return 6650.0, 'fallback'


class Clocks:
    """nvidia-smi sampler started before and stopped after the timed region."""
    QUERY = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
             'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
             'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu_id):
        self.gpu_id, self.proc, self.path = gpu_id, None, None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix='.csv')
        os.close(fd)
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={self.QUERY}', '--format=csv,noheader,nounits',
                                          '-i', str(self.gpu_id), '-lms', '100'],
                                         stdout=open(self.path, 'w'), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        self.proc.wait(timeout=10)
        rows = []
        for line in Path(self.path).read_text().splitlines():
            f = [x.strip() for x in line.split(',')]
            if len(f) >= 9 and f[1].isdigit():
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [int(r[1]) for r in rows]
        reasons = set()
        for r in rows:
            for name, col in [('hw_slowdown', 5), ('hw_thermal_slowdown', 6), ('sw_thermal_slowdown', 7),
                              ('sw_power_cap', 8)]:
                if r[col].lower() == 'active':
                    reasons.add(name)
        loaded = [s for s in sm if s > 0.5 * max(sm)]
        return {'sm_mhz': int(statistics.median(loaded or sm)), 'sm_max_mhz': int(rows[0][2]),
                'samples': len(rows), 'reasons': sorted(reasons)}


def dist_setup():
    import torch
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device('cuda', local))
    return rank, world, local


def max_over_ranks(value, world):
    if world == 1:
        return value
    from qwen_b200.distributed import reduce_over_ranks
    return reduce_over_ranks(value, 'max')


def barrier(world):
    import torch
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def oracle_batch(seqs, context, extra, threads):
    """The oracle (plain-C port of the reference's behavioural model, KV8
    mode) holding `seqs` sequences at contexts `context`..`context`+4 with the
    seeded synthetic caches of the GPU arm. Its assets come from the oracle's
    own link of the seeded generator (no product library is loaded)."""
    from oracle import ref
    with tempfile.TemporaryDirectory() as tmp:
        ref.synth_write(tmp, SEED)
        m = ref.RefModel(tmp, capacity=context + 8 + extra, mode=ref.KV8, threads=threads)
    m.set_slots(seqs)
    for s in range(seqs):
        m.fill_kv_synthetic_slot(s, context + s % 5, SEED + 17 * s)
    return m


def cpu_decode_sample(seqs, context, min_seconds, max_seconds, threads):
    """Batched decode steps of `seqs` sequences on the host cores (each step
    one forward of seqs rows, weights streamed once), for min..max seconds.
    Returns (tokens/s, steps timed)."""
    m = oracle_batch(seqs, context, 64, threads)
    slots = np.arange(seqs, dtype=np.uint32)
    toks = np.random.default_rng(SEED).integers(0, VOCAB, seqs).astype(np.uint32)
    toks, _ = m.decode_batch(slots, toks)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        toks, _ = m.decode_batch(slots, toks)
        n += 1
        el = time.perf_counter() - t0
        if (el >= min_seconds and n >= 2) or el >= max_seconds or n >= 60:
            break
    m.close()
    return seqs * n / el, n


def run_reference(args):
    """The CPU reference of the path (the oracle port: the reference's model
    is Python over torch and its C code holds no model math) on the same
    workload as the GPU arm: one step = one greedy decode step of args.seqs
    sequences at context args.context+, as one batched forward."""
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    m = oracle_batch(args.seqs, args.context, args.steps + args.warmup, threads)
    slots = np.arange(args.seqs, dtype=np.uint32)
    toks = np.random.default_rng(SEED).integers(0, VOCAB, args.seqs).astype(np.uint32)
    for _ in range(args.warmup):
        toks, _ = m.decode_batch(slots, toks)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        toks, _ = m.decode_batch(slots, toks)
    el = time.perf_counter() - t0
    m.close()
    value = args.seqs * args.steps / el
    sample = (f'oracle/qwen_ref.c (KV8 mode, the reference model\'s arithmetic) decoding {args.seqs} sequences '
              f'at context {args.context}..{args.context + 4}+ as one batched forward per step, '
              f'{args.steps} steps after {args.warmup} warm-up, {threads} OpenMP threads')
    cfg = workload_config(args)
    cfg['global_batch'] = args.seqs  # rank 0 alone runs the CPU arm
    cfg['parallelism'] = 'one host process (rank 0), all host cores'
    line = {'metric': 'decode tokens/s', 'value': round(value, 3), 'unit': 'tokens/s', 'impl': 'reference',
            'n_gpus': args.gpus, 'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': round(1000 * el / args.steps, 3), 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'int8 weights x bf16 activations, fp32 accumulate, int8 KV',
            'data': 'synthetic (seeded random-init int8 weights, seeded KV8 fill, random token ids)',
            'config': cfg,
            'cpu_baseline': {'value': round(value, 3), 'unit': 'tokens/s', 'cores': threads, 'kind': 'port',
                             'sample': sample},
            'e2e': {'value': round(value, 3), 'unit': 'tokens/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)
    return 0


def workload_config(args):
    return {'workload': f'batched greedy decode, {args.seqs} sequences per GPU at context {args.context}+, '
                        'Qwen2.5-0.5B W8A16 with KV8 cache',
            'model': 'Qwen2.5-0.5B (24 layers, hidden 896, seeded random int8 weights)',
            'seqs_per_gpu': args.seqs, 'global_batch': args.seqs * args.gpus, 'context': args.context,
            'contexts': f'{args.context}..{args.context + 4} at the first timed step (sequence s at '
                        f'{args.context} + s % 5)',
            'parallelism': f'request-sharded replicas x{args.gpus} (no inter-GPU traffic)',
            'l2': 'inputs larger than L2 (weights 496 MB + KV ~0.88 GB per step)'}


def run_ours(args):
    import torch
    import qwen_b200
    rank, world, local = dist_setup()
    torch.cuda.set_device(local)
    if args.steps + args.warmup > 120:
        raise SystemExit('--steps + --warmup must stay within one 128-key context bucket (<= 120)')
    S, C = args.seqs, args.context
    cap = C + 2 * (args.steps + args.warmup) + 64
    eng = qwen_b200.Engine(device=local, max_seqs=S, max_context=cap, max_rows=256).load_synthetic(SEED)

    def fill(n):
        # contexts C..C+4 (ragged), the caches of the oracle's batched step
        for s in range(n):
            eng.fill_kv_synthetic(s, C + s % 5, SEED + 17 * s + rank)

    fill(S)
    rng = np.random.default_rng(SEED + rank)
    first = rng.integers(0, VOCAB, S).astype(np.int32)
    bufs = [torch.tensor(first, device='cuda'), torch.zeros(S, dtype=torch.int32, device='cuda')]
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)

    def step(i):
        a, b = bufs[i % 2], bufs[(i + 1) % 2]
        eng.decode_step_device(ctypes.c_void_p(a.data_ptr()), S, ctypes.c_void_p(b.data_ptr()), sp)

    for i in range(args.warmup):
        step(i)
    contexts0 = [eng.position(s) + 1 for s in range(S)]
    barrier(world)
    clocks = Clocks(gpu_index(local))
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        step(args.warmup + i)
    t1.record(stream)
    barrier(world)
    clk = clocks.stop()
    ms = t0.elapsed_time(t1)
    ms_max = max_over_ranks(ms, world)
    launches = qwen_b200.lib().qwen_b200_step_launches(eng.h) * args.steps
    value = world * S * args.steps / (ms_max / 1000.0)
    contexts = [c + args.steps // 2 for c in contexts0]  # mean context over the timed steps
    sbytes = step_bytes(contexts)
    hbm, peak_kind = peaks()

    # e2e: the same step through the host-buffer C ABI call
    toks = bufs[args.warmup % 2].cpu().numpy().astype(np.uint32)
    slots = np.arange(S, dtype=np.uint32)
    for _ in range(2):
        toks = eng.decode_step(slots, toks)
    barrier(world)
    e0 = time.perf_counter()
    for _ in range(args.steps):
        toks = eng.decode_step(slots, toks)
    e_s = max_over_ranks(time.perf_counter() - e0, world)
    e2e = {'value': round(world * S * args.steps / e_s, 1), 'unit': 'tokens/s',
           'h2d_bytes_per_step': 3 * 4 * S, 'd2h_bytes_per_step': 4 * S,
           'api': 'qwen_b200_decode_step (host buffers)'}

    # per-kernel-class device times of a real step (events on the launching stream)
    ms_cls = np.zeros(len(CLASSES), np.float32)
    n_cls = np.zeros(len(CLASSES), np.uint32)
    out = np.empty(S, np.uint32)
    for rep in range(2):
        rc = qwen_b200.lib().qwen_b200_profile_decode(
            eng.h, toks.ctypes.data_as(qwen_b200._lib._P32), S, out.ctypes.data_as(qwen_b200._lib._P32),
            ms_cls.ctypes.data_as(qwen_b200._lib._PF), n_cls.ctypes.data_as(qwen_b200._lib._P32))
        assert rc == 0, qwen_b200.lib().qwen_b200_last_error(eng.h)
        toks = out.copy()
    prof_ctx = [eng.position(s) for s in range(S)]
    cb = class_bytes(S, prof_ctx)
    kernels = {}
    for i, name in enumerate(CLASSES):
        if n_cls[i]:
            per = float(ms_cls[i]) / int(n_cls[i])
            kernels[name] = {'launches_per_step': int(n_cls[i]), 'ms_per_step': round(float(ms_cls[i]), 4),
                             'us_per_launch': round(1000 * per, 2),
                             'gbs': round(cb[name] / (per / 1000) / 1e9, 1)}
    dom = max(kernels, key=lambda k: kernels[k]['ms_per_step'])
    dom_us = kernels[dom]['us_per_launch']
    achieved = cb[dom] / (dom_us / 1e6) / 1e9
    roofline = {'kernel': kernel_names(S)[dom], 'class': dom, 'bound': 'hbm', 'achieved': round(achieved, 1),
                'peak': hbm, 'peak_kind': peak_kind, 'unit': 'GB/s', 'frac': round(achieved / hbm, 4),
                'algorithmic_bytes_per_launch': cb[dom], 'traffic': committed_traffic(dom),
                'traffic_source': ('ncu dram__bytes_read.sum + dram__bytes_write.sum of this kernel class at this '
                                   'workload, from the committed capture summarised in profiles/traffic.json '
                                   '(not measured in this run)') if committed_traffic(dom) else None}
    step_ms = ms_max / args.steps
    step_roof = {'bytes_per_step': sbytes, 'achieved': round(sbytes / (step_ms / 1000) / 1e9, 1), 'peak': hbm,
                 'unit': 'GB/s', 'frac': round(sbytes / (step_ms / 1000) / 1e9 / hbm, 4)}

    # fixed global batch (strong scaling): the same 64 sequences split over
    # the ranks, 64 / N per GPU; each GPU still streams every weight per step
    strong = strong_scaling(eng, args, world, value, step_ms_of(ms_max, args), fill, stream, sp)

    # bs1 decode at short context (16-token prompt), slot 0
    bs1 = bs1_decode(eng, args, stream, sp, hbm)
    eng.close()

    # prefill of 8 x 4096-token prompts with the vocabulary-sharded LM head
    prefill = None if args.no_prefill else prefill_sharded(args, rank, world, local)

    result = None
    if rank == 0:
        result = {
            'metric': 'decode tokens/s', 'value': round(value, 1), 'unit': 'tokens/s', 'n_gpus': world,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(step_ms, 4),
            'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
            'dtype': 'int8 weights x bf16 activations, fp32 accumulate, int8 KV',
            'data': 'synthetic (seeded random-init int8 weights, seeded KV8 fill, random token ids)',
            'config': workload_config(args), 'roofline': roofline, 'step_roofline': step_roof,
            'kernels': kernels, 'e2e': e2e, 'gpu_launches': int(launches), 'bs1': bs1, 'strong': strong,
            'prefill': prefill, 'clocks': clk}
    if world == 1 and not args.no_cpu_baseline:
        tps, n = cpu_decode_sample(S, C, 10.0, 30.0, os.cpu_count() or 1)
        result['cpu_baseline'] = {'value': round(tps, 3), 'unit': 'tokens/s', 'cores': os.cpu_count() or 1,
                                  'kind': 'port',
                                  'sample': f'oracle/qwen_ref.c (KV8 mode) decoding {S} sequences at context '
                                            f'{C}..{C + 4}+, {n} batched steps (one {S}-row forward each)'}
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)
    return 0


def prefill_sharded(args, rank, world, local):
    """Prefill of args.prefill_prompts prompts of args.prefill_len seeded random
    ids through all 24 layers (tensor-core projections; the rows of all of a
    GPU's prompts go through the layers together, --prefill-chunk at a time),
    request-sharded (prompts / N per GPU), then the LM head split by
    vocabulary over the GPUs: an NCCL all-gather of every prompt's last hidden
    row, each GPU's (value, index) per row over its vocabulary range, an NCCL
    all-gather of those candidates and the highest-value / highest-index
    combine (model_backend.py:113-114). Timed on the host around the whole
    sequence (the prefill call synchronises), max over ranks."""
    import torch
    import qwen_b200
    import qwen_b200.distributed as D
    P, T = args.prefill_prompts, args.prefill_len
    if P % world:
        return {'unavailable': f'{P} prompts do not split evenly over {world} GPUs'}
    mine = list(D.shard_requests(P, world, rank))
    rng = np.random.default_rng(SEED + 99)
    prompts = [rng.integers(0, VOCAB, T).astype(np.uint32) for _ in range(P)]  # the same on every rank
    eng = qwen_b200.Engine(device=local, max_seqs=P, max_context=T + 8,
                           max_rows=args.prefill_chunk).load_synthetic(SEED)
    vb, ve = D.vocab_shard(VOCAB, world, rank)
    # bf16 bit patterns, gathered as bfloat16 (NCCL has no 16-bit integer type)
    hid_local = torch.empty((len(mine), HID), dtype=torch.bfloat16, device='cuda')
    hid_all = torch.empty((P, HID), dtype=torch.bfloat16, device='cuda')
    vals = torch.empty(P, dtype=torch.float32, device='cuda')
    idx = torch.empty(P, dtype=torch.int32, device='cuda')
    vals_all = torch.empty(world * P, dtype=torch.float32, device='cuda')
    idx_all = torch.empty(world * P, dtype=torch.int32, device='cuda')
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)

    def run():
        for s in mine:
            eng.reset(s)
        _, hidden = eng.prefill(mine, [prompts[i] for i in mine], want_tokens=False, want_hidden=True)
        hid_local.copy_(torch.from_numpy(hidden.view(np.int16)).view(torch.bfloat16))
        if world > 1:
            import torch.distributed as dist
            dist.all_gather_into_tensor(hid_all, hid_local)
        else:
            hid_all.copy_(hid_local)
        eng.lm_head_range(ctypes.c_void_p(hid_all.data_ptr()), P, vb, ve, ctypes.c_void_p(vals.data_ptr()),
                          ctypes.c_void_p(idx.data_ptr()), sp)
        if world > 1:
            import torch.distributed as dist
            dist.all_gather_into_tensor(vals_all, vals)
            dist.all_gather_into_tensor(idx_all, idx)
        else:
            vals_all.copy_(vals)
            idx_all.copy_(idx)
        return D.combine_candidates(vals_all.cpu().numpy().reshape(world, P),
                                    idx_all.cpu().numpy().reshape(world, P).astype(np.int64))

    tokens = run()  # warm-up (captures nothing: prefill launches directly)
    times = []
    for _ in range(args.prefill_reps):
        barrier(world)
        t0 = time.perf_counter()
        tokens = run()
        torch.cuda.synchronize()
        times.append(max_over_ranks(time.perf_counter() - t0, world))
    # the sharded head agrees with each rank's own full-vocabulary head
    for s in mine:
        eng.reset(s)
    own, _ = eng.prefill(mine, [prompts[i] for i in mine], want_tokens=True, want_hidden=False)
    agree = reduce_agree(bool(np.array_equal(own.astype(np.int64), tokens[mine])), world)
    eng.close()
    sec = min(times)
    return {'metric': 'prefill tokens/s', 'value': round(P * T / sec, 1), 'unit': 'tokens/s',
            'ms_per_run': round(1000 * sec, 2), 'runs': args.prefill_reps, 'prompts': P, 'prompt_len': T,
            'prompts_per_gpu': len(mine), 'vocab_shard_rows': ve - vb,
            'collectives': ('NCCL all-gather of the last hidden rows, then of the per-shard (value, index)'
                            if world > 1 else 'none (one GPU holds the whole vocabulary)'),
            'sharded_tokens_equal_full_head': agree,
            'timing': 'host wall clock around the synchronous prefill call, gathers and sharded LM head, '
                      'max over ranks, best of the runs'}


def reduce_agree(flag, world):
    return bool(reduce_over_ranks_min(1.0 if flag else 0.0, world) == 1.0)


def reduce_over_ranks_min(value, world):
    if world == 1:
        return value
    from qwen_b200.distributed import reduce_over_ranks
    return -reduce_over_ranks(-value, 'max')


def step_ms_of(ms_max, args):
    return ms_max / args.steps


# HBM-roofline ceiling of a fixed global batch of 64 at context 2048 split
# over N GPUs (every GPU streams the 496 MB of weights each step), relative
# to one GPU: roofline tokens/s ratios 1, 1.47, 1.92, 2.27.
STRONG_CEILING = {1: 1.0, 2: 1.47, 4: 1.92, 8: 2.27}


def strong_scaling(eng, args, world, value, step_ms, fill, stream, sp):
    """Fixed global batch: args.seqs sequences over all ranks (seqs / N per
    GPU), timed like the main step (device events, max over ranks)."""
    import torch
    S = args.seqs
    if world == 1:
        return {'global_batch': S, 'seqs_per_gpu': S, 'value': round(value, 1), 'ms_per_step': round(step_ms, 4),
                'roofline_ceiling_vs_1gpu': 1.0, 'note': 'one GPU: the main measurement'}
    if S % world:
        return {'global_batch': S, 'unavailable': f'{S} sequences do not split evenly over {world} GPUs'}
    n = S // world
    fill(n)  # slots 0..n-1 back at contexts C..C+4
    bufs = [torch.randint(0, VOCAB, (n,), dtype=torch.int32, device='cuda'),
            torch.zeros(n, dtype=torch.int32, device='cuda')]

    def step(i):
        eng.decode_step_device(ctypes.c_void_p(bufs[i % 2].data_ptr()), n,
                               ctypes.c_void_p(bufs[(i + 1) % 2].data_ptr()), sp)

    for i in range(args.warmup):
        step(i)
    barrier(world)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        step(args.warmup + i)
    t1.record(stream)
    barrier(world)
    ms_max = max_over_ranks(t0.elapsed_time(t1), world)
    return {'global_batch': S, 'seqs_per_gpu': n, 'value': round(world * n * args.steps / (ms_max / 1000.0), 1),
            'ms_per_step': round(ms_max / args.steps, 4),
            'roofline_ceiling_vs_1gpu': STRONG_CEILING.get(world)}


def bs1_decode(eng, args, stream, sp, hbm):
    import torch
    prompt = np.zeros(16, np.uint32)
    import qwen_b200
    qwen_b200.lib().qwen_b200_synth_prompt(SEED, 16, prompt.ctypes.data_as(qwen_b200._lib._P32))
    eng.reset(0)
    tok, _ = eng.forward(0, prompt, 0)
    a = torch.tensor([tok], dtype=torch.int32, device='cuda')
    b = torch.zeros(1, dtype=torch.int32, device='cuda')
    bufs = [a, b]
    for i in range(args.warmup):
        eng.decode_step_device(ctypes.c_void_p(bufs[i % 2].data_ptr()), 1,
                               ctypes.c_void_p(bufs[(i + 1) % 2].data_ptr()), sp)
    ctx0 = eng.position(0) + 1
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(args.steps):
        j = args.warmup + i
        eng.decode_step_device(ctypes.c_void_p(bufs[j % 2].data_ptr()), 1,
                               ctypes.c_void_p(bufs[(j + 1) % 2].data_ptr()), sp)
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    sb = step_bytes([ctx0 + args.steps // 2])
    ach = sb / (ms / 1000) / 1e9
    # device time per kernel class of one bs1 step (events around each launch)
    ms_cls = np.zeros(len(CLASSES), np.float32)
    n_cls = np.zeros(len(CLASSES), np.uint32)
    tok_in = np.array([int(bufs[(args.warmup + args.steps) % 2][0].item())], np.uint32)
    out = np.empty(1, np.uint32)
    qwen_b200.lib().qwen_b200_profile_decode(eng.h, tok_in.ctypes.data_as(qwen_b200._lib._P32), 1,
                                             out.ctypes.data_as(qwen_b200._lib._P32),
                                             ms_cls.ctypes.data_as(qwen_b200._lib._PF),
                                             n_cls.ctypes.data_as(qwen_b200._lib._P32))
    kernels = {name: {'launches': int(n_cls[i]), 'us_per_step': round(1000 * float(ms_cls[i]), 1)}
               for i, name in enumerate(CLASSES) if n_cls[i]}
    return {'value': round(1000 / ms, 1), 'unit': 'tokens/s', 'ms_per_token': round(ms, 4),
            'context': ctx0 + args.steps // 2, 'bytes_per_token': sb, 'achieved_gbs': round(ach, 1),
            'frac_of_hbm_roofline': round(ach / hbm, 4), 'kernels': kernels,
            'kernel_sum_us': round(1000 * float(ms_cls.sum()), 1)}


def gpu_index(local):
    vis = os.environ.get('CUDA_VISIBLE_DEVICES')
    if vis:
        ids = [v.strip() for v in vis.split(',') if v.strip()]
        if local < len(ids):
            return ids[local]
    return local


def committed_traffic(cls):
    """DRAM bytes per launch from the committed ncu summary, if one exists for
    this kernel class at this workload (profiles/traffic.json)."""
    p = REPO / 'profiles' / 'traffic.json'
    if not p.exists():
        return None
    return json.loads(p.read_text()).get(cls)


# The operator microbenchmarks: the model's projection shapes [K x N] at
# M rows, and KV8 GQA decode attention at context L for B rows.
GEMM_SHAPES = [('qkv', HID, QKV, 'bias'), ('o', HID, HID, 'residual'), ('gate_up', HID, 2 * FFN, 'swiglu'),
               ('down', FFN, HID, 'residual'), ('lm_head', HID, VOCAB, 'argmax')]
GEMM_ROWS = [1, 8, 64, 512, 4096]
ATTN_CONTEXTS = [512, 2048, 8192, 32768]
ATTN_BATCHES = [1, 16, 64]
INT8_DENSE_NOMINAL = 4.5e15  # int8 tensor ops/s, dense, nominal


def micro_timer(torch, stream, reps):
    """Median CUDA-event time (us) of one launch of fn after an L2 flush
    (a 256 MB write, larger than the 126 MB L2) before every timed launch."""
    flush = torch.empty(256 << 20, dtype=torch.uint8, device='cuda')

    def run(fn):
        for _ in range(3):
            assert fn() == 0
        times = []
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            rc = fn()
            e1.record(stream)
            assert rc == 0, rc
            e1.synchronize()
            times.append(1000.0 * e0.elapsed_time(e1))
        return statistics.median(times)
    return run


def micro_gemm(torch, L, stream, sp, timed, hbm):
    """W8A16 projections through the C ABI, on the kernel family the engine
    runs at that row count: one row on the GEMV family (qwen_b200_op_gemm_w8a16
    / _residual, op_swiglu, op_lm_head_argmax), two rows and more on the
    tcgen05 GEMM (qwen_b200_op_gemm_w8a16_tc, which also builds the activation
    limb planes; the LM head shape writes its bf16 logits). Weights int8
    per-output-channel from N(0, 0.02), activations bf16 N(0, 1)."""
    g = torch.Generator(device='cuda').manual_seed(SEED)
    out = []
    for name, K, N, epi in GEMM_SHAPES:
        wf = torch.randn(N, K, device='cuda', generator=g) * 0.02
        scale = (wf.abs().amax(1) / 127).clamp_min(1e-12)
        w = torch.round(wf / scale[:, None]).clamp(-127, 127).to(torch.int8).contiguous()
        scale = scale.to(torch.bfloat16).float().contiguous()
        del wf
        bias = (torch.randn(N, device='cuda', generator=g) * 0.02).to(torch.bfloat16)
        for M in GEMM_ROWS:
            x = torch.randn(M, K, device='cuda', generator=g).to(torch.bfloat16)
            n_out = N // 2 if epi == 'swiglu' else N
            y = torch.zeros(M, n_out, device='cuda', dtype=torch.bfloat16)
            ws = None
            if M == 1:
                if epi == 'argmax':
                    wsb = L.qwen_b200_lm_head_workspace(M, N)
                    ws = torch.zeros(wsb, dtype=torch.uint8, device='cuda')
                    tok = torch.zeros(M, dtype=torch.int32, device='cuda')
                    fn = lambda: L.qwen_b200_op_lm_head_argmax(x.data_ptr(), M, None, 1e-6, w.data_ptr(),
                                                               scale.data_ptr(), N, None, tok.data_ptr(),
                                                               ws.data_ptr(), wsb, sp)
                    kernel = 'lm_head1_kernel + argmax_reduce_kernel'
                elif epi == 'swiglu':
                    fn = lambda: L.qwen_b200_op_swiglu(x.data_ptr(), M, None, 1e-6, w.data_ptr(), scale.data_ptr(),
                                                       y.data_ptr(), sp)
                    kernel = 'gemv_kernel<896,EPI_SWIGLU>'
                elif epi == 'residual':
                    fn = lambda: L.qwen_b200_op_gemm_w8a16_residual(x.data_ptr(), M, K, w.data_ptr(),
                                                                    scale.data_ptr(), N, y.data_ptr(), sp)
                    kernel = f'gemv_kernel<{K},EPI_RESIDUAL>'
                else:
                    fn = lambda: L.qwen_b200_op_gemm_w8a16(x.data_ptr(), M, K, w.data_ptr(), scale.data_ptr(), N,
                                                           bias.data_ptr(), y.data_ptr(), sp)
                    kernel = f'gemv_kernel<{K},EPI_BIAS>'
            else:
                code = {'bias': 1, 'residual': 2, 'swiglu': 3, 'argmax': 0}[epi]
                wsb = L.qwen_b200_gemm_tc_workspace(M, N, K)
                ws = torch.zeros(wsb, dtype=torch.uint8, device='cuda')
                fn = lambda: L.qwen_b200_op_gemm_w8a16_tc(x.data_ptr(), M, K, w.data_ptr(), scale.data_ptr(), N,
                                                          bias.data_ptr() if code == 1 else None, code, y.data_ptr(),
                                                          ws.data_ptr(), wsb, sp)
                kernel = 'act_quant_kernel + tc_gemm_kernel'
            us = timed(fn)
            if M > 1:
                assert int(ws[:4].view(torch.int32)[0].item()) == 0, 'pipeline wait expired'
            out_bytes = (0 if epi == 'argmax' and M == 1 else M * n_out * 2) * (2 if epi == 'residual' else 1)
            nbytes = N * K + 4 * N + (2 * N if epi == 'bias' else 0) + M * K * 2 + out_bytes
            flops = 2.0 * M * N * K
            rec = {'shape': f'{K}x{N}', 'name': name, 'rows': M, 'kernel': kernel, 'us': round(us, 2),
                   'bytes': nbytes, 'gbs': round(nbytes / us / 1e3, 1), 'hbm_frac': round(nbytes / us / 1e3 / hbm, 4),
                   'tops': round(flops / us / 1e6, 2)}
            if M > 1:
                # exact mode: four int8 limb planes, i.e. 4 x 2MNK tensor ops executed
                rec['int8_tensor_frac_nominal'] = round(4 * flops / (us * 1e-6) / INT8_DENSE_NOMINAL, 4)
            out.append(rec)
            del x, y, ws
        del w, scale, bias
        torch.cuda.empty_cache()
    return out


def attention_kernel_name(rows, keys, max_splits=16):
    """The kernel the engine's attention launch picks (the split plan of
    attention_rs.cu; 16-way clusters where the GPU places them)."""
    chunks = -(-keys // 192)
    s = max(min(148 // (2 * rows), max_splits, chunks), 1, -(-chunks // 12))
    if s > max_splits or (s > 8 and rows * 2 * s > 4 * 148):
        return 'attn_cluster_kernel'
    return 'attn_rs_kernel'


def micro_attention(torch, L, stream, sp, timed, hbm):
    """KV8 GQA decode attention (qwen_b200_op_attention_cluster, the engine's
    form): B rows, each in its own slot at context L (keys 0..L-1); K and V
    drawn bf16 N(0, 1), RoPE applied to K (qwen_b200_op_rope), quantised per
    token and head by qwen_b200_op_kv8_append; q bf16 N(0, 1)."""
    g = torch.Generator(device='cuda').manual_seed(SEED + 1)
    out = []
    for C in ATTN_CONTEXTS:
        table_h = (ctypes.c_float * (C * 64))()
        L.qwen_b200_rope_table(C, table_h)
        table = torch.tensor(np.frombuffer(table_h, dtype=np.float32), device='cuda')
        for B in ATTN_BATCHES:
            rows = B * C
            slots = torch.arange(B, dtype=torch.int32, device='cuda').repeat_interleave(C)
            pos = torch.arange(C, dtype=torch.int32, device='cuda').repeat(B)
            kc = torch.empty(B, 2, C, 64, dtype=torch.int8, device='cuda')
            vc = torch.empty_like(kc)
            ks = torch.empty(B, 2, C, dtype=torch.float32, device='cuda')
            vs = torch.empty_like(ks)
            for codes, scales, rope in ((kc, ks, True), (vc, vs, False)):
                raw = torch.randn(rows, 2, 64, device='cuda', generator=g).to(torch.bfloat16)
                if rope:
                    assert L.qwen_b200_op_rope(raw.data_ptr(), rows, 2, pos.data_ptr(), table.data_ptr(), sp) == 0
                assert L.qwen_b200_op_kv8_append(raw.data_ptr(), rows, slots.data_ptr(), pos.data_ptr(),
                                                 codes.data_ptr(), scales.data_ptr(), C, sp) == 0
                del raw
            q = torch.randn(B, 14, 64, device='cuda', generator=g).to(torch.bfloat16)
            ctx = torch.zeros(B, HID, dtype=torch.bfloat16, device='cuda')
            qs = torch.arange(B, dtype=torch.int32, device='cuda')
            qp = torch.full((B,), C - 1, dtype=torch.int32, device='cuda')
            fn = lambda: L.qwen_b200_op_attention_cluster(q.data_ptr(), B, qs.data_ptr(), qp.data_ptr(), C,
                                                          kc.data_ptr(), ks.data_ptr(), vc.data_ptr(), vs.data_ptr(),
                                                          C, ctx.data_ptr(), sp)
            us = timed(fn)
            nbytes = B * C * KV_BYTES_PER_TOKEN_LAYER + B * HID * 2 * 2
            out.append({'context': C, 'batch': B, 'kernel': attention_kernel_name(B, C),
                        'us': round(us, 2), 'bytes': nbytes, 'gbs': round(nbytes / us / 1e3, 1),
                        'hbm_frac': round(nbytes / us / 1e3 / hbm, 4)})
            del kc, vc, ks, vs, q, ctx, slots, pos
            torch.cuda.empty_cache()
    return out


def micro_prefill_attention(torch, L, stream, sp, timed):
    """Attention of one 4096-token prompt's rows (positions 0..4095 of one
    slot, causal): the query-tiled tensor-core kernel
    (qwen_b200_op_attention_prefill, the engine's prefill form) against the
    per-row kernel (qwen_b200_op_attention_cluster) on the same rows; both
    give the same bits. Codes uniform in [-127, 127], scales in [0, 0.02], q
    bf16 N(0, 1)."""
    T = 4096
    cap = T + 8
    g = torch.Generator(device='cuda').manual_seed(SEED + 2)
    kc = torch.randint(-127, 128, (2, cap, 64), dtype=torch.int8, device='cuda', generator=g)
    vc = torch.randint(-127, 128, (2, cap, 64), dtype=torch.int8, device='cuda', generator=g)
    ks = torch.rand(2, cap, device='cuda', generator=g) * 0.02
    vs = torch.rand(2, cap, device='cuda', generator=g) * 0.02
    q = torch.randn(T, 14, 64, device='cuda', generator=g).to(torch.bfloat16)
    ctx_t = torch.zeros(T, HID, dtype=torch.bfloat16, device='cuda')
    ctx_r = torch.zeros_like(ctx_t)
    slots = torch.zeros(T, dtype=torch.int32, device='cuda')
    pos = torch.arange(T, dtype=torch.int32, device='cuda')
    wsb = L.qwen_b200_attention_prefill_workspace(T)
    ws = torch.zeros(wsb, dtype=torch.uint8, device='cuda')
    tiled = lambda: L.qwen_b200_op_attention_prefill(q.data_ptr(), T, 0, kc.data_ptr(), ks.data_ptr(), vc.data_ptr(),
                                                     vs.data_ptr(), cap, ctx_t.data_ptr(), ws.data_ptr(), wsb, sp)
    per_row = lambda: L.qwen_b200_op_attention_cluster(q.data_ptr(), T, slots.data_ptr(), pos.data_ptr(), T,
                                                       kc.data_ptr(), ks.data_ptr(), vc.data_ptr(), vs.data_ptr(), cap,
                                                       ctx_r.data_ptr(), sp)
    us_t = timed(tiled)
    us_r = timed(per_row)
    assert int(ws[:4].view(torch.int32)[0].item()) == 0, 'a bounded wait expired'
    elements = T * (T + 1) // 2 * 14
    return {'rows': T, 'positions': '0..4095 of one slot', 'tiled_us': round(us_t, 1), 'per_row_us': round(us_r, 1),
            'tiled_kernel': 'attn_tile_kernel', 'per_row_kernel': attention_kernel_name(T, T),
            'same_bits': bool(torch.equal(ctx_t, ctx_r)),
            'row_head_key_elements': elements, 'tiled_g_elements_per_s': round(elements / us_t / 1e3, 1)}


def run_micro(args):
    import torch
    import qwen_b200
    torch.cuda.set_device(0)
    L = qwen_b200.lib()
    stream = torch.cuda.current_stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    hbm, peak_kind = peaks()
    timed = micro_timer(torch, stream, args.micro_reps)
    clocks = Clocks(gpu_index(0))
    clocks.start()
    part = args.micro_part
    gemm = micro_gemm(torch, L, stream, sp, timed, hbm) if part in ('all', 'gemm') else None
    attn = micro_attention(torch, L, stream, sp, timed, hbm) if part in ('all', 'attention') else None
    pre = micro_prefill_attention(torch, L, stream, sp, timed) if part in ('all', 'prefill') else None
    clk = clocks.stop()
    print(json.dumps({'record': 'operator microbenchmarks', 'n_gpus': 1, 'hbm_peak_gbs': hbm,
                      'peak_kind': peak_kind, 'reps': args.micro_reps,
                      'timing': 'median of per-launch CUDA events on the launching stream, L2 flushed '
                                '(256 MB write) before every timed launch, after 3 warm-up launches',
                      'gemm': gemm, 'attention': attn, 'prefill_attention': pre, 'clocks': clk}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=30)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', choices=['ours', 'reference'], default='ours')
    ap.add_argument('--seqs', type=int, default=64)
    ap.add_argument('--context', type=int, default=2048)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-prefill', action='store_true')
    ap.add_argument('--prefill-prompts', type=int, default=8)
    ap.add_argument('--prefill-len', type=int, default=4096)
    ap.add_argument('--prefill-reps', type=int, default=2)
    ap.add_argument('--prefill-chunk', type=int, default=32768,
                    help='rows that go through the layers together (the engine\'s max_rows)')
    ap.add_argument('--prefill-only', action='store_true',
                    help='run only the prefill record (prints its own JSON object)')
    ap.add_argument('--micro', action='store_true',
                    help='run only the operator microbenchmarks (projection shapes x rows, attention '
                         'contexts x batches; one GPU; prints its own JSON object)')
    ap.add_argument('--micro-reps', type=int, default=20)
    ap.add_argument('--micro-part', choices=['all', 'gemm', 'attention', 'prefill'], default='all')
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit('--warmup must be >= 3')
    if args.impl == 'reference':
        return run_reference(args)
    if args.micro:
        return run_micro(args)
    if args.prefill_only:
        import torch
        rank, world, local = dist_setup()
        torch.cuda.set_device(local)
        rec = prefill_sharded(args, rank, world, local)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(rec), flush=True)
        return 0
    return run_ours(args)


if __name__ == '__main__':
    sys.exit(main())
