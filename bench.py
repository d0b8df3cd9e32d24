"""Benchmark of the ASRN layer forward on B200 (the metric of BASELINE.json):

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Workload (configuration 3 of the benchmark, the layer metric): one ASRNLayer(768) forward with default options on
32 sequences x 8192 tokens per GPU, fp32 E/h as the model passes them, bf16 autocast; tokens Zipf(1.1) over 50,304
with 20 % of positions in planted repeats of length 16-256 (seeded synthetic data, asrn_b200/synthetic.py), E rows from
a random embedding table, random-init weights with the neutral parameters moved off zero. A step is one layer forward
over the GPU's batch. Batches shard across GPUs with no collective, so per-GPU work is fixed (weak scaling).

Printed (rank 0, one JSON line): value = tokens/s of the whole job (all ranks' tokens / max-over-ranks device time of
K steps, inputs resident in HBM; the 805 MB E and h per GPU exceed the 126 MB L2, so no flush is needed), e2e = the
same through ASRNLayer.forward with pinned host buffers and H2D/D2H copies in the timed region, roofline of the
dominant kernel (candidate scoring, HBM-bound), the CPU baseline (the oracle port on the host cores), clocks (nvidia-smi
samples inside the timed region; the sampler starts before the warm-up). Warm-up: at least W steps, then until two
consecutive steps agree within 3 % (at most 20 more; "warmup" reports the count); then the forward is captured once as a
CUDA graph and the K timed steps are its replays ("launch": "cuda_graph"; --eager times the eager forward; the
sequence-sharded cfg4 forward with its NCCL collectives stays eager); "step_ms" gives the spread of the K timed steps
(CUDA events between them).
Generation leg (configuration 5, key "generation"): the configuration-3 model (random init), 64 sequences split over
the GPUs with 65,536-token Zipf+repeat prompts, then greedy steps of the O(1) writer; value = device time per step
(us per generated token of every sequence), with the same figure at 4,096 and 16,384-token prompts (flatness), the
prefill rate, and the public generate() API end to end.
--impl reference: times the CPU implementation of the path (oracle port) on the host cores instead.
"""
import argparse
import datetime
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

D, L_SEQ, B_PER_GPU, V = 768, 8192, 32, 50304
METRIC = 'asrn_layer_fwd_tokens_per_s'
UNIT = 'tokens/s'
# Algorithmic HBM bytes per token of the candidate-scoring kernel at this config (bf16 features, fp32 accumulator):
# per table, a key's phi + Kc + query phi + Qc (2 * 128 * 2 B), its value row (768 * 2 B) and 72 B of ids / clock /
# log_alfa / signature; plus the output row (768 * 2 B): T * (512 + 1536 + 72) + 1536 = 18,496 B.
SCORE_BYTES_PER_TOKEN = 8 * (2 * 128 * 2 + D * 2 + 72) + D * 2
LAYER_BYTES_PER_TOKEN = 34696
# generation leg (configuration 5): the configuration-3 model, 64 sequences split over the GPUs, 65,536-token prompts,
# greedy steps; flatness is checked at shorter prompts too
GEN_B, GEN_L0, GEN_NEW, GEN_FLAT = 64, 65536, 1024, (4096, 16384)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=20)
    p.add_argument('--warmup', type=int, default=3)
    p.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    p.add_argument('--batch', type=int, default=B_PER_GPU, help='sequences per GPU')
    p.add_argument('--seq', type=int, default=L_SEQ)
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--workload', default='cfg3', choices=['cfg3', 'cfg4'],
                   help='cfg3: the batch-sharded layer metric (default); cfg4: one 262,144-token sequence, d=512, '
                        'sequence-sharded over the GPUs')
    p.add_argument('--no-gen', action='store_true', help='skip the generation leg')
    p.add_argument('--eager', action='store_true', help='time the eager forward instead of its CUDA-graph replay')
    p.add_argument('--gen-prompt', type=int, default=GEN_L0, help='prompt length of the generation leg')
    p.add_argument('--gen-steps', type=int, default=GEN_NEW, help='timed generation steps')
    return p.parse_args()


def config(args, n):
    return {'workload': 'cfg3 layer: ASRNLayer(768) forward, %d x %d tokens per GPU, bf16 autocast, fp32 E/h'
                        % (args.batch, args.seq),
            'global_batch': args.batch * n, 'seq_len': args.seq, 'd': D, 'vocab': V,
            'parallelism': 'dp%d (batch sharded, no collective)' % n,
            'l2': 'inputs larger than L2 (E and h are %.0f MB each per GPU; L2 is 126 MB), no flush'
                  % (args.batch * args.seq * D * 4 / 1e6)}


# ---------------------------------------------------------------------------------------------------------------------
# inputs
# ---------------------------------------------------------------------------------------------------------------------

def make_layer_params(seed=0, d=D):
    """Random-init ASRNLayer(d) weights with the neutral (zero-init) parameters moved off zero (the reference tests'
    recipe)."""
    import torch
    import asrn_b200
    torch.manual_seed(seed)
    layer = asrn_b200.ASRNLayer(d)
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for n, p in layer.named_parameters():
            if n in ('w_reloj', 'b_reloj', 'gamma', 'log_kappa', 'log_kappa_racha', 'u_hawkes', 'd_racha', 'cq.weight',
                     'w_sufijo', 'w_vistos', 'g_conf.weight', 'g_conf.bias'):
                p.add_(torch.randn(p.shape, generator=g) * 0.5)
        layer.gamma.copy_(torch.linspace(0.5, 3.0, layer.n_tablas))
    return layer


def make_inputs(batch, seq, rank, seed=0):
    """(tokens int64 (B, L), E float32 (B, L, d), h float32 (B, L, d)) as numpy; rank-dependent seeds."""
    import numpy as np
    from asrn_b200 import synthetic
    x = synthetic.config_tokens('cfg3', B=batch, L=seq, seed=seed + 1000 * rank)
    g = np.random.default_rng(seed + 7)
    table = (g.standard_normal((V, D)) * 0.02).astype(np.float32)      # emb init std 0.02 (asrn/nucleo.py:1066)
    E = table[x]
    h = (E + g.standard_normal(E.shape).astype(np.float32) * 0.5).astype(np.float32)
    return x, E, h, table


# ---------------------------------------------------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------------------------------------------------


def graph_or_eager(step, eager):
    """The forward captured once as a CUDA graph after the warm-up (only on paths with no collective): the K timed
    steps are then K graph launches, all enqueued ahead of the device, so a host-side pause cannot leave the GPU idle
    between steps; the kernels and their work are those of the eager forward. Returns (run, mode, graph)."""
    import torch
    if eager:
        return step, 'eager', None
    try:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        graph.replay()
        return graph.replay, 'cuda_graph', graph
    except Exception as exc:              # capture unsupported here: time the eager forward
        return step, 'eager (graph capture failed: %s)' % type(exc).__name__, None

class ClockSampler:
    """nvidia-smi clock / throttle-reason samples every 100 ms. Started before the warm-up (nvidia-smi's own start-up
    then happens outside the timed region); mark() brackets the timed region, and only samples inside it count."""
    FIELDS = ('timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.f = None
        self.window = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile('w+', suffix='.csv', delete=False)
            self.proc = subprocess.Popen(['nvidia-smi', '-i', str(self.idx), '--query-gpu=' + self.FIELDS,
                                          '--format=csv,noheader,nounits', '-lms', '100'], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        # wait (up to 10 s) for the first sample: nvidia-smi is up before the GPU work that is measured
        t_end = time.time() + 10
        while time.time() < t_end and os.path.getsize(self.f.name) == 0 and self.proc.poll() is None:
            time.sleep(0.05)

    def mark(self, t0, t1):
        """The timed region in host wall-clock seconds (time.time())."""
        self.window = (t0, t1)

    def stop(self):
        if self.proc is None:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['nvidia-smi unavailable']}
        time.sleep(0.15)                      # one more sample after the timed region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [r.split(',') for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        parsed = []
        for r in rows:
            try:
                ts = datetime.datetime.strptime(r[0].strip(), '%Y/%m/%d %H:%M:%S.%f').timestamp()
                parsed.append((ts, r))
            except (ValueError, IndexError):
                continue
        inside = parsed
        if self.window is not None:
            lo, hi = self.window
            sel = [(ts, r) for ts, r in parsed if lo - 0.1 <= ts <= hi + 0.1]
            inside = sel if sel else parsed
        sm, mx, reasons = [], [], set()
        names = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')
        for _, r in inside:
            try:
                sm.append(float(r[2]))
                mx.append(float(r[3]))
                for nm, v in zip(names, r[6:10]):
                    if v.strip().lower() in ('active', '1'):
                        reasons.add(nm)
            except (ValueError, IndexError):
                continue
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': max(mx) if mx else None,
                'reasons': sorted(reasons), 'samples': len(sm)}


def warm_up(step, warmup, world):
    """At least max(3, warmup) untimed steps; then, up to 20 more, until two consecutive steps agree within 3 % (the
    first steps of a process run slower while allocations and the GPU's clocks settle). All ranks take the same number
    of steps (the slowest rank's count decides). Returns the number of warm-up steps taken."""
    import torch
    n = 0
    times = []
    while True:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
        n += 1
        settled = n >= max(3, warmup) and (n >= max(3, warmup) + 20 or
                                           abs(times[-1] - times[-2]) <= 0.03 * min(times[-1], times[-2]))
        if world > 1:
            import torch.distributed as dist
            flag = torch.tensor([0 if settled else 1], device='cuda')
            dist.all_reduce(flag)
            settled = flag.item() == 0
        if settled:
            return n


# ---------------------------------------------------------------------------------------------------------------------
# CPU baseline: the oracle port (the reference's algorithm restated in numpy) on the host cores
# ---------------------------------------------------------------------------------------------------------------------

def _oracle_one(payload):
    """One sequence through the oracle's vectorised layer forward; returns seconds. Runs in a spawned worker."""
    os.environ.setdefault('OMP_NUM_THREADS', '1')
    os.environ.setdefault('OPENBLAS_NUM_THREADS', '1')
    import numpy as np
    sys.path.insert(0, HERE)
    from oracle import asrn_oracle as O
    params, x, E, h = payload
    lay = O.Layer(params, E.shape[-1])
    t0 = time.perf_counter()
    O.layer_forward_fast(lay, E, h, x, half=True)
    return time.perf_counter() - t0


def host_cores():
    """Host cores this process may use: the affinity mask, capped by a cgroup CPU quota if one is set."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, 'sched_getaffinity') else (os.cpu_count() or 1)
    try:
        with open('/sys/fs/cgroup/cpu.max') as f:
            quota, period = f.read().split()
        if quota != 'max':
            n = min(n, max(1, int(int(quota) / int(period))))
    except (OSError, ValueError):
        pass
    return max(1, n)


def cpu_baseline(layer_params, x, E, h, seq, workers=None):
    """Tokens/s of the oracle port on `workers` host processes (one sequence each, spawn pool)."""
    import multiprocessing as mp
    workers = workers or max(1, min(host_cores(), x.shape[0], 32))
    ctx = mp.get_context('spawn')
    n = min(workers, x.shape[0])
    payloads = [(layer_params, x[i:i + 1, :seq], E[i:i + 1, :seq], h[i:i + 1, :seq]) for i in range(n)]
    # one BLAS thread per worker process: the workers import numpy while unpickling their task, so the limit has to be
    # in the environment they inherit (16 workers x 16 BLAS threads each oversubscribe the cores 16 times)
    saved = {k: os.environ.get(k) for k in ('OMP_NUM_THREADS', 'OPENBLAS_NUM_THREADS', 'MKL_NUM_THREADS')}
    os.environ.update({k: '1' for k in saved})
    try:
        with ctx.Pool(n) as pool:
            pool.map(_oracle_one, payloads[:n])          # warm-up: imports, first-touch of the arrays
            t0 = time.perf_counter()
            secs = pool.map(_oracle_one, payloads)
            wall = time.perf_counter() - t0
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    tok = n * seq
    return {'value': tok / wall, 'unit': UNIT, 'cores': n, 'kind': 'port',
            'sample': '%d sequence(s) x %d tokens of the same workload, one per host process (numpy oracle port of '
                      'the reference CPU path, bf16 autocast emulated); wall %.1f s, per-sequence %.1f s'
                      % (n, seq, wall, statistics.median(secs))}


# ---------------------------------------------------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------------------------------------------------

def dist_env():
    rank = int(os.environ.get('RANK', 0))
    world = int(os.environ.get('WORLD_SIZE', 1))
    local = int(os.environ.get('LOCAL_RANK', 0))
    return rank, world, local


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    import numpy as np
    import torch
    layer = make_layer_params()
    params = {k: v.detach().numpy() for k, v in layer.state_dict().items()}
    seq = args.seq
    x, E, h, _ = make_inputs(max(1, min(32, host_cores())), seq, 0)
    vals = []
    info = None
    for _ in range(max(1, min(args.steps, 3))):
        info = cpu_baseline(params, x, E, h, seq)
        vals.append(info['value'])
    v = statistics.median(vals)
    info['value'] = v
    out = {'metric': METRIC, 'value': v, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
           'ms_per_step': None, 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None, 'dtype': 'bf16',
           'data': 'synthetic', 'impl': 'reference', 'config': config(args, world), 'cpu_baseline': info,
           'e2e': {'value': v, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(out), flush=True)
    return 0


def load_profile_traffic():
    """Per-launch DRAM bytes of the scoring kernel from the committed ncu summary (profiles/), or None."""
    p = os.path.join(HERE, 'profiles', 'k_score_tc_cfg3_traffic.json')
    try:
        with open(p) as f:
            t = json.load(f)
        return t.get('dram_bytes_per_token')
    except (OSError, ValueError):
        return None


def run_generation(args, dev, rank, world):
    """Generation leg: per prompt length, the prompt pass (prefill) then args.gen_steps greedy steps of the O(1)
    writer, each step the CUDA-graph replay of the model's step plus a device argmax feeding the next token (no host
    sync), timed with CUDA events; then the public API (generate, top_k=1) end to end at the shortest prompt."""
    import torch
    import asrn_b200
    from asrn_b200 import synthetic
    B = max(1, GEN_B // world)
    torch.manual_seed(0)
    m = asrn_b200.create_model(V=V, d=D, n_capas=12, semilla=0).to(dev).eval()
    prompts = sorted(set([p for p in GEN_FLAT if p < args.gen_prompt] + [args.gen_prompt]))
    out = {'sequences_per_gpu': B, 'prompts': {}}
    for L0 in prompts:
        x0 = torch.from_numpy(synthetic.config_tokens('cfg5', B=B, L=L0, seed=rank)).to(dev)
        with torch.autocast('cuda', dtype=torch.bfloat16):
            w = asrn_b200.Writer(m)
            torch.cuda.synchronize()
            p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            p0.record()
            lg = w.inicio(x0, capacidad=L0 + args.gen_steps + 8)
            p1.record()
            nxt = lg.argmax(-1)
            for _ in range(3):
                nxt = w.paso(nxt, copiar=False).argmax(-1)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.gen_steps):
                nxt = w.paso(nxt, copiar=False).argmax(-1)
            e1.record()
            torch.cuda.synchronize()
            status = w.status()
            if any(status):
                raise RuntimeError(f'generation step status {status}')
            out['prompts'][str(L0)] = {'step_us': e0.elapsed_time(e1) / args.gen_steps * 1e3,
                                       'prefill_tokens_per_s': B * L0 / (p0.elapsed_time(p1) * 1e-3)}
            w.cerrar()
            del w, lg, nxt, x0
        torch.cuda.empty_cache()
    # public API end to end (host tokens in, host tokens out, sampling as the reference's): per-token cost from two
    # calls that differ only in the number of new tokens
    L0 = prompts[0]
    x0 = torch.from_numpy(synthetic.config_tokens('cfg5', B=B, L=L0, seed=rank))
    n_a, n_b = 8, 72
    times = []
    with torch.autocast('cuda', dtype=torch.bfloat16):
        asrn_b200.generate(m, x0, n_nuevos=4, top_k=1, devolver_logits=False)
        for n in (n_a, n_b):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            asrn_b200.generate(m, x0, n_nuevos=n, top_k=1, devolver_logits=False)
            torch.cuda.synchronize()
            times.append(time.perf_counter() - t0)
    out['e2e_step_us'] = (times[1] - times[0]) / (n_b - n_a) * 1e6
    out['e2e_prompt'] = L0
    del m
    torch.cuda.empty_cache()
    return out


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    rank, world, local = dist_env()
    if world > 1:
        import datetime
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    import asrn_b200
    from asrn_b200 import stages

    layer = make_layer_params().to(dev).eval()
    x_np, E_np, h_np, _table = make_inputs(args.batch, args.seq, rank)
    cpu_info = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        params = {k: v.detach().cpu().numpy() for k, v in layer.state_dict().items()}
        cpu_info = cpu_baseline(params, x_np, E_np, h_np, args.seq)
    x = torch.from_numpy(x_np).to(dev)
    E = torch.from_numpy(E_np).to(dev)
    h = torch.from_numpy(h_np).to(dev)
    tokens = args.batch * args.seq

    def step():
        with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
            return layer(E, h, x)

    clocks = ClockSampler(local)
    clocks.start()
    warm = warm_up(step, args.warmup, world)
    run, launch_mode, graph = graph_or_eager(step, args.eager)
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    gc.collect()
    gc.disable()                  # no collector pause while the steps are enqueued
    torch.cuda.synchronize()
    w0 = time.time()
    t0.record()
    for i in range(args.steps):
        run()
        marks[i].record()
    t1.record()
    torch.cuda.synchronize()
    gc.enable()
    clocks.mark(w0, time.time())
    ms = t0.elapsed_time(t1)
    step_ms = [t0.elapsed_time(marks[0])] + [marks[i - 1].elapsed_time(marks[i]) for i in range(1, args.steps)]
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    # launches of our kernels per forward: context, clock, hash, bucket sort (1, or 3 when rows span tiles),
    # scoring, n-gram rows, streak, gate prep, gate
    launches_per_step = 8 + (1 if args.seq <= 8192 else 3)

    # dominant kernel (candidate scoring), timed on its launching stream with the forward's own intermediates
    with torch.no_grad():
        ctx = stages.context(layer, h, x, half=True)
        Bt = stages.clock(ctx['beta'])
        hs = stages.hash(layer, E, half=True)
        orden, ids_o = stages.bucket_sort(hs['ids_rows'], layer.n_bits)
        call = lambda: stages.score(layer, orden, ids_o, hs['phi'], ctx['Qc'], ctx['Kc'], ctx['sig'], Bt,
                                    ctx['log_alfa'], hs['Ea'], half=True)
        for _ in range(2):
            call()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(args.steps):
            call()
        s1.record()
        torch.cuda.synchronize()
        score_ms = s0.elapsed_time(s1) / args.steps
        del ctx, Bt, hs, orden, ids_o

    # end to end through the public API with pinned host buffers
    Eh = torch.from_numpy(E_np).pin_memory()
    hh = torch.from_numpy(h_np).pin_memory()
    xh = torch.from_numpy(x_np).pin_memory()
    out_h = torch.empty_like(hh).pin_memory()

    def e2e_step():
        Ed, hd, xd = Eh.to(dev, non_blocking=True), hh.to(dev, non_blocking=True), xh.to(dev, non_blocking=True)
        with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
            yd = layer(Ed, hd, xd)
        out_h.copy_(yd, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_steps = max(2, min(args.steps, 5))
    e0.record()
    for _ in range(e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e_steps

    del Eh, hh, xh, out_h, E, h, x, run, graph
    torch.cuda.empty_cache()
    gen = None
    if not args.no_gen:
        gen = run_generation(args, dev, rank, world)
    g_step = [gen['prompts'][k]['step_us'] for k in sorted(gen['prompts'], key=int)] if gen else []
    vals = [ms, e2e_ms, score_ms] + g_step + ([gen['e2e_step_us']] if gen else [])
    times = torch.tensor(vals, device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    vals = times.tolist()
    ms, e2e_ms, score_ms = vals[:3]
    if gen:
        for k, v in zip(sorted(gen['prompts'], key=int), vals[3:3 + len(g_step)]):
            gen['prompts'][k]['step_us'] = v
        gen['e2e_step_us'] = vals[-1]
    if rank == 0:
        import json as _json
        peaks = {}
        try:
            with open(os.path.join(HERE, 'MEASURED_PEAKS.json')) as f:
                peaks = _json.load(f)
        except (OSError, ValueError):
            pass
        hbm = peaks.get('hbm_gbs', 6650.0)
        peak_src = 'measured' if 'hbm_gbs' in peaks else 'fallback'
        achieved = SCORE_BYTES_PER_TOKEN * tokens / (score_ms * 1e-3) / 1e9
        traffic_pt = load_profile_traffic()
        value = world * tokens * args.steps / (ms * 1e-3)
        out = {'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
               'warmup': warm, 'ms_per_step': ms / args.steps,
               'step_ms': {'min': min(step_ms), 'median': statistics.median(step_ms), 'max': max(step_ms),
                           'argmax': step_ms.index(max(step_ms))},
               'higher_is_better': True,
               'scaling': 'weak', 'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic',
               'config': config(args, world),
               'e2e': {'value': world * tokens / (e2e_ms * 1e-3), 'unit': UNIT,
                       'h2d_bytes_per_step': int(E_np.nbytes + h_np.nbytes + x_np.nbytes),
                       'd2h_bytes_per_step': int(h_np.nbytes)},
               'roofline': {'bound': 'hbm', 'kernel': 'k_score (candidate scoring)', 'achieved': achieved,
                            'peak': hbm, 'peak_source': peak_src, 'unit': 'GB/s', 'frac': achieved / hbm,
                            'algorithmic_bytes_per_token': SCORE_BYTES_PER_TOKEN,
                            'traffic': None if traffic_pt is None else traffic_pt * tokens,
                            'kernel_ms': score_ms,
                            'layer_frac': LAYER_BYTES_PER_TOKEN * tokens / (ms / args.steps * 1e-3) / 1e9 / hbm},
               'gpu_launches': launches_per_step * args.steps,
               'launch': launch_mode,
               'clocks': clk}
        if cpu_info is not None:
            out['cpu_baseline'] = cpu_info
        if gen:
            main = gen['prompts'][str(args.gen_prompt)]
            out['generation'] = {
                'metric': 'gen_us_per_token', 'value': main['step_us'], 'unit': 'us/token', 'higher_is_better': False,
                'workload': 'cfg5: create_model(V=50304, d=768, n_capas=12) random init, %d sequences (%d per GPU), '
                            'Zipf+repeat prompts of %d tokens, %d greedy steps (CUDA-graph step + device argmax), '
                            'bf16 autocast' % (gen['sequences_per_gpu'] * world, gen['sequences_per_gpu'],
                                               args.gen_prompt, args.gen_steps),
                'step_us_by_prompt': {k: v['step_us'] for k, v in gen['prompts'].items()},
                'prefill_tokens_per_s_by_prompt': {k: v['prefill_tokens_per_s'] * world
                                                   for k, v in gen['prompts'].items()},
                'tokens_per_s': gen['sequences_per_gpu'] * world / (main['step_us'] * 1e-6),
                'e2e': {'value': gen['e2e_step_us'], 'unit': 'us/token',
                        'api': 'asrn_b200.generate(top_k=1, devolver_logits=False), host prompt of %d tokens; '
                               'per-token cost = difference of a 72- and an 8-token call / 64' % gen['e2e_prompt']}}
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


D4, L4 = 512, 262144
CFG4_BYTES_PER_TOKEN = 24968     # algorithmic HBM bytes per token of one layer forward at d=512, bf16, fp32 E/h


def run_cfg4(args):
    """Configuration 4: one sequence of L4 tokens, ASRNLayer(512), bf16 autocast, sequence-sharded over the GPUs
    (asrn_b200.shard: halo + clock-offset + feature all-gathers over NCCL); strong scaling. value = tokens of the
    sequence per second (max-over-ranks device time of a step, exchange included)."""
    import datetime
    import numpy as np
    import torch
    import torch.distributed as dist
    rank, world, local = dist_env()
    if world > 1:
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    from asrn_b200 import shard, synthetic
    L = args.seq if args.seq != L_SEQ else L4
    layer = make_layer_params(d=D4).to(dev).eval()
    x = synthetic.config_tokens('cfg4', B=1, L=L, seed=0)
    g = np.random.default_rng(7)
    table = (g.standard_normal((V, D4)) * 0.02).astype(np.float32)
    c0, c1 = shard.chunk_bounds(L, world, rank)
    xc = np.ascontiguousarray(x[:, c0:c1])
    Ec = table[xc]
    hc = (Ec + np.random.default_rng(8 + rank).standard_normal(Ec.shape).astype(np.float32) * 0.5).astype(np.float32)
    cpu_info = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        seg = 16384
        nseg = max(1, min(host_cores(), L // seg, 16))
        params = {k: v.detach().cpu().numpy() for k, v in layer.state_dict().items()}
        xs = x[:, :nseg * seg].reshape(nseg, seg)
        Es = table[xs]
        hs = (Es + np.random.default_rng(9).standard_normal(Es.shape).astype(np.float32) * 0.5).astype(np.float32)
        cpu_info = cpu_baseline(params, xs, Es, hs, seg)
        cpu_info['sample'] = ('%d segments of %d tokens of the sequence, each run as its own sequence, one per host '
                              'process (numpy oracle port, bf16 autocast emulated)' % (nseg, seg))
    xd, Ed, hd = (torch.from_numpy(a).to(dev) for a in (xc, Ec, hc))

    def step():
        with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
            if world == 1:
                return layer(Ed, hd, xd)
            return shard.forward(layer, Ed, hd, xd)

    clocks = ClockSampler(local)
    clocks.start()
    warm = warm_up(step, args.warmup, world)
    # one GPU: the forward replayed as a CUDA graph; sharded: eager (its NCCL collectives stay outside graphs)
    run, launch_mode, graph = graph_or_eager(step, args.eager or world > 1)
    if world > 1:
        dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    gc.collect()
    gc.disable()                  # no collector pause while the steps are enqueued
    torch.cuda.synchronize()
    w0 = time.time()
    t0.record()
    for i in range(args.steps):
        run()
        marks[i].record()
    t1.record()
    torch.cuda.synchronize()
    gc.enable()
    clocks.mark(w0, time.time())
    ms = t0.elapsed_time(t1)
    step_ms = [t0.elapsed_time(marks[0])] + [marks[i - 1].elapsed_time(marks[i]) for i in range(1, args.steps)]
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    # end to end: this rank's chunk from pinned host buffers, h' back to the host
    xh, Eh, hh = (torch.from_numpy(a).pin_memory() for a in (xc, Ec, hc))
    out_h = torch.empty(hh.shape, dtype=torch.float32).pin_memory()

    def e2e_step():
        xe, Ee, he = xh.to(dev, non_blocking=True), Eh.to(dev, non_blocking=True), hh.to(dev, non_blocking=True)
        with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
            ye = layer(Ee, he, xe) if world == 1 else shard.forward(layer, Ee, he, xe)
        out_h.copy_(ye, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_steps = max(2, min(args.steps, 5))
    e0.record()
    for _ in range(e_steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e_steps
    times = torch.tensor([ms, e2e_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, e2e_ms = times.tolist()
    if rank == 0:
        peaks = {}
        try:
            with open(os.path.join(HERE, 'MEASURED_PEAKS.json')) as f:
                peaks = json.load(f)
        except (OSError, ValueError):
            pass
        hbm = peaks.get('hbm_gbs', 6650.0)
        step_s = ms / args.steps * 1e-3
        achieved = CFG4_BYTES_PER_TOKEN * (L // world) / step_s / 1e9
        out = {'metric': METRIC, 'value': L / step_s, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
               'warmup': warm, 'ms_per_step': ms / args.steps,
               'step_ms': {'min': min(step_ms), 'median': statistics.median(step_ms), 'max': max(step_ms),
                           'argmax': step_ms.index(max(step_ms))},
               'higher_is_better': True,
               'scaling': 'strong', 'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic',
               'config': {'workload': 'cfg4 layer: ASRNLayer(512) forward, 1 x %d tokens, bf16 autocast, fp32 E/h'
                                      % L, 'global_batch': 1, 'seq_len': L, 'd': D4, 'vocab': V,
                          'parallelism': ('sequence-sharded over %d GPUs (NCCL all-gathers of the halo, clock '
                                          'offsets, bucket tails, per-position features, n-gram summaries and '
                                          'streak maps)' % world) if world > 1 else 'single GPU',
                          'l2': 'inputs larger than L2 (E and h are %.0f MB each per GPU), no flush'
                                % (Ec.nbytes / 1e6)},
               'e2e': {'value': L / (e2e_ms * 1e-3), 'unit': UNIT, 'h2d_bytes_per_step': int(xc.nbytes + Ec.nbytes +
                                                                                             hc.nbytes),
                       'd2h_bytes_per_step': int(hc.nbytes)},
               'roofline': {'bound': 'hbm', 'kernel': 'whole layer forward (per GPU)', 'achieved': achieved,
                            'peak': hbm, 'peak_source': 'measured' if 'hbm_gbs' in peaks else 'fallback',
                            'unit': 'GB/s', 'frac': achieved / hbm,
                            'algorithmic_bytes_per_token': CFG4_BYTES_PER_TOKEN, 'traffic': None},
               'gpu_launches': None, 'launch': launch_mode, 'clocks': clk}
        if cpu_info is not None:
            out['cpu_baseline'] = cpu_info
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == 'reference':
        return run_reference(args)
    if args.workload == 'cfg4':
        return run_cfg4(args)
    return run_ours(args)


if __name__ == '__main__':
    sys.exit(main())
