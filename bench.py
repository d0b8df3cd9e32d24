"""Benchmark of the ASRN layer forward on B200 (the metric of BASELINE.json):

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Headline workload (configuration 3 of the benchmark, the layer metric): one ASRNLayer(768) forward with default options
on 32 sequences x 8192 tokens per GPU, fp32 E/h as the model passes them, bf16 autocast; tokens Zipf(1.1) over 50,304
with 20 % of positions in planted repeats of length 16-256 (seeded synthetic data, asrn_b200/synthetic.py), E rows from
a random embedding table (std 0.02, the model's initialisation), random-init weights with the neutral parameters moved
off zero. A step is one layer forward over the GPU's batch. Batches shard across GPUs with no collective, so per-GPU
work is fixed (weak scaling).

Printed (rank 0, one JSON line):
  value      tokens/s of the whole job: all ranks' tokens / the max-over-ranks device time of K steps, inputs resident
             in HBM (the 805 MB E and h per GPU exceed the 126 MB L2, so no flush is needed). After the warm-up the
             forward is captured once as a CUDA graph and the K timed steps are its replays.
  e2e        the same through ASRNLayer.forward from pinned host buffers: every step copies its E, h and tokens to the
             device and h' back, on copy streams that overlap step k's compute with step k+1's upload and step k-1's
             download (PCIe is full duplex).
  roofline   the dominant kernel (candidate scoring, HBM-bound): its algorithmic bytes per launch / its CUDA-event
             launch time, against the measured HBM peak (MEASURED_PEAKS.json); traffic from the committed ncu summary.
  cpu_baseline  the reference's own CPU implementation (asrn.ASRNLayer installed into baseline/_ref, PyTorch on the
             host cores) on a bounded sample of the same workload.
  gpu_launches  kernel nodes of the captured forward (ours are named k_*) x K.
  clocks     nvidia-smi samples inside the timed region.
Legs in the same line (each with its own value, device timing and the reference's CPU time beside it):
  generation configuration 5: the configuration-3 model, 64 sequences split over the GPUs, 65,536-token Zipf+repeat
             prompts, greedy steps of the O(1) writer (CUDA-graph step + asrn_argmax_rows); flatness at 4,096 and 16,384;
             the public generate() end to end; the reference's _Escritor(o1=True) at batch 4 on the host cores.
  cfg4       one 262,144-token sequence, ASRNLayer(512), bf16: one GPU, or sequence-sharded over the GPUs of the run
             (NCCL exchanges of halo, clock offsets, bucket tails, features, n-gram summaries and streak maps).
  cfg2       ASRNLayer(256) forward in fp32, 16 x 4096 tokens (batch-sharded).
  cfg1       create_model(V=256, d=64, n_capas=4) forward on 8 x 256 bytes, then generate(top_k=1) of 200 tokens.
  model      the configuration-3 model forward (shared n-gram sort, fused local blocks) on 4 x 8192 tokens.
  train      ASRNLayer(768) forward + backward in training mode, bf16 autocast, 4 x 8192 tokens (rank 0), beside the
             reference's forward + backward on the host cores.
--impl reference: times the reference's CPU implementation of the headline workload (asrn.ASRNLayer from
baseline/_ref, torch on the host cores, bf16 autocast, chunks of 4 sequences per step) and its O(1) writer.
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
REF_PATH = os.path.join(HERE, 'baseline', '_ref')

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
D4, L4 = 512, 262144
CFG4_BYTES_PER_TOKEN = 24968     # algorithmic HBM bytes per token of one layer forward at d=512, bf16, fp32 E/h
D2, B2, L2 = 256, 16, 4096
CFG2_BYTES_PER_TOKEN = 25256     # d=256, fp32
REF_CHUNK = 4                    # sequences per step of the reference's CPU timing (its V_o buffer is ~6.5 GB per 4)
TRAIN_B = 4                      # sequences of the training leg (cfg3 shapes: ASRNLayer(768), 8192 tokens, bf16)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument('--gpus', type=int, default=1)
    p.add_argument('--steps', type=int, default=20)
    p.add_argument('--warmup', type=int, default=3)
    p.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    p.add_argument('--batch', type=int, default=B_PER_GPU, help='sequences per GPU')
    p.add_argument('--seq', type=int, default=L_SEQ)
    p.add_argument('--no-cpu-baseline', action='store_true')
    p.add_argument('--workload', default='cfg3', choices=['cfg3', 'cfg4', 'gen', 'model', 'localblock', 'train'],
                   help='cfg3: the batch-sharded layer metric (default); cfg4 / gen / model / localblock / train: '
                        'only that leg (for profiling)')
    p.add_argument('--no-gen', action='store_true', help='skip the generation leg')
    p.add_argument('--no-legs', action='store_true', help='skip the cfg1 / cfg2 / cfg4 legs')
    p.add_argument('--eager', action='store_true', help='time the eager forward instead of its CUDA-graph replay')
    p.add_argument('--gen-prompt', type=int, default=GEN_L0, help='prompt length of the generation leg')
    p.add_argument('--gen-steps', type=int, default=GEN_NEW, help='timed generation steps')
    p.add_argument('--gen-cpu-prompts', default='4096',
                   help='prompt lengths of the reference writer on the host (comma list; 16384 and 65536 take minutes)')
    return p.parse_args()


def config(args, n):
    return {'workload': 'cfg3 layer: ASRNLayer(768) forward, %d x %d tokens per GPU, bf16 autocast, fp32 E/h'
                        % (args.batch, args.seq),
            'global_batch': args.batch * n, 'seq_len': args.seq, 'd': D, 'vocab': V,
            'parallelism': 'dp%d (batch sharded, no collective)' % n,
            'l2': 'inputs larger than L2 (E and h are %.0f MB each per GPU; L2 is 126 MB), no flush'
                  % (args.batch * args.seq * D * 4 / 1e6)}


def peaks():
    try:
        with open(os.path.join(HERE, 'MEASURED_PEAKS.json')) as f:
            p = json.load(f)
    except (OSError, ValueError):
        p = {}
    return p.get('hbm_gbs', 6650.0), ('measured' if 'hbm_gbs' in p else 'fallback')


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


def make_cfg4_inputs(L, c0, c1, rank):
    import numpy as np
    from asrn_b200 import synthetic
    x = synthetic.config_tokens('cfg4', B=1, L=L, seed=0)
    table = (np.random.default_rng(7).standard_normal((V, D4)) * 0.02).astype(np.float32)
    xc = np.ascontiguousarray(x[:, c0:c1])
    Ec = table[xc]
    hc = (Ec + np.random.default_rng(8 + rank).standard_normal(Ec.shape).astype(np.float32) * 0.5).astype(np.float32)
    return x, xc, Ec, hc, table


def make_cfg2_inputs(batch, rank):
    import numpy as np
    from asrn_b200 import synthetic
    x = synthetic.config_tokens('cfg2', B=batch, L=L2, seed=1000 * rank)
    g = np.random.default_rng(20 + rank)
    E = g.standard_normal((batch, L2, D2)).astype(np.float32)
    h = g.standard_normal((batch, L2, D2)).astype(np.float32)
    return x, E, h


# ---------------------------------------------------------------------------------------------------------------------
# clocks during the timed region, warm-up, graph capture
# ---------------------------------------------------------------------------------------------------------------------

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


def _kernel_node_name(nd):
    """Name of a graph kernel node's function (driver API, then runtime API), or '?'."""
    try:
        from cuda.bindings import driver as cu
        err, prm = cu.cuGraphKernelNodeGetParams(cu.CUgraphNode(int(nd)))
        if int(err) == 0:
            err, nm = cu.cuFuncGetName(prm.func)
            if int(err) == 0:
                return nm.decode() if isinstance(nm, bytes) else str(nm)
    except Exception:
        pass
    try:
        from cuda.bindings import runtime as rt
        err, prm = rt.cudaGraphKernelNodeGetParams(nd)
        err, nm = rt.cudaFuncGetName(prm.func)
        if int(err) == 0:
            return nm.decode() if isinstance(nm, bytes) else str(nm)
    except Exception:
        pass
    return '?'


def count_graph_kernels(graph):
    """(all kernel nodes, those of libasrn_b200 (named k_*), {name: count}) of a captured CUDA graph, or Nones."""
    try:
        from cuda.bindings import runtime as rt
        g = graph.raw_cuda_graph()
        err, _, n = rt.cudaGraphGetNodes(g, 0)
        err, nodes, n = rt.cudaGraphGetNodes(g, n)
        kernels, ours, names = 0, 0, {}
        for nd in nodes:
            err, ty = rt.cudaGraphNodeGetType(nd)
            if ty != rt.cudaGraphNodeType.cudaGraphNodeTypeKernel:
                continue
            kernels += 1
            name = _kernel_node_name(nd)
            short = name.split('(')[0].split('<')[0].replace('asrn::', '')
            names[short] = names.get(short, 0) + 1
            if 'asrn' in name or short.startswith('k_') or short.startswith('_ZN4asrn'):
                ours += 1
        return kernels, ours, names
    except Exception:
        return None, None, None


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
        graph = torch.cuda.CUDAGraph(keep_graph=True)
        with torch.cuda.graph(graph):
            step()
        graph.instantiate()
        graph.replay()
        return graph.replay, 'cuda_graph', graph
    except Exception as exc:              # capture unsupported here: time the eager forward
        return step, 'eager (graph capture failed: %s)' % type(exc).__name__, None


def timed(run, steps, clocks=None, barrier=False):
    """K back-to-back steps between two CUDA events on the current stream: (total ms, per-step ms list). barrier:
    every rank calls this, and the ranks meet at a barrier after the collector ran and the device went idle, so the
    first step's collectives do not wait for a rank still collecting."""
    import torch
    import torch.distributed as dist
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    gc.collect()
    gc.disable()                  # no collector pause while the steps are enqueued
    torch.cuda.synchronize()
    if barrier and dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
        torch.cuda.synchronize()
    w0 = time.time()
    t0.record()
    for i in range(steps):
        run()
        marks[i].record()
    t1.record()
    torch.cuda.synchronize()
    gc.enable()
    if clocks is not None:
        clocks.mark(w0, time.time())
    step_ms = [t0.elapsed_time(marks[0])] + [marks[i - 1].elapsed_time(marks[i]) for i in range(1, steps)]
    return t0.elapsed_time(t1), step_ms


def spread(step_ms):
    return {'min': min(step_ms), 'median': statistics.median(step_ms), 'max': max(step_ms),
            'argmax': step_ms.index(max(step_ms))}


def e2e_pipelined(forward, host_in, host_out, dev, steps):
    """Public-API throughput from pinned host buffers: step k uploads its inputs on a copy stream while step k-1
    computes, and downloads its h' on a second copy stream while step k+1 computes (two device buffer sets). Returns
    ms per step (CUDA events around all the copies and forwards)."""
    import torch
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    bufs = [[torch.empty(t.shape, dtype=t.dtype, device=dev) for t in host_in] for _ in range(2)]
    outs = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (host_out, host_out)]
    uploaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]

    def upload(k):
        i = k % 2
        with torch.cuda.stream(s_in):
            s_in.wait_event(consumed[i])
            for dst, src in zip(bufs[i], host_in):
                dst.copy_(src, non_blocking=True)
            uploaded[i].record(s_in)

    def run(n):
        upload(0)
        for k in range(n):
            i = k % 2
            comp.wait_event(uploaded[i])
            y = forward(*bufs[i])
            consumed[i].record(comp)
            computed[i].record(comp)
            if k + 1 < n:
                upload(k + 1)
            with torch.cuda.stream(s_out):
                s_out.wait_event(computed[i])
                outs[i].copy_(y, non_blocking=True)
                y.record_stream(s_out)
        comp.wait_stream(s_out)
        comp.wait_stream(s_in)

    run(2)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    run(steps)
    e1.record(comp)
    torch.cuda.synchronize()
    host_out.copy_(outs[(steps - 1) % 2])
    return e0.elapsed_time(e1) / steps


# ---------------------------------------------------------------------------------------------------------------------
# the reference's own CPU implementation (installed into baseline/_ref)
# ---------------------------------------------------------------------------------------------------------------------

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


def import_reference():
    """The reference package (KIROKOWA/ASRN) as pip installed it into baseline/_ref; ImportError if absent."""
    if not os.path.isdir(os.path.join(REF_PATH, 'asrn')):
        raise ImportError('baseline/_ref/asrn is not installed')
    if REF_PATH not in sys.path:
        sys.path.insert(0, REF_PATH)
    import asrn
    if not os.path.abspath(asrn.__file__).startswith(os.path.abspath(REF_PATH)):
        raise ImportError('asrn resolves to %s, not baseline/_ref' % asrn.__file__)
    return asrn


def ref_layer_steps(state, x, E, h, half, per_step, steps, warmup):
    """The reference's ASRNLayer forward on the host (torch CPU, all granted cores), `per_step` sequences per step
    cycling over the sample: per-step seconds of `steps` timed steps after `warmup`."""
    import torch
    asrn = import_reference()
    torch.set_num_threads(host_cores())
    d = E.shape[-1]
    layer = asrn.ASRNLayer(d)
    layer.load_state_dict(state)
    layer.eval()
    xs, Es, hs = (torch.from_numpy(a) for a in (x, E, h))
    n = x.shape[0]
    secs = []
    for i in range(warmup + steps):
        b0 = (i * per_step) % n
        sl = slice(b0, min(n, b0 + per_step))
        t0 = time.perf_counter()
        with torch.no_grad(), torch.autocast('cpu', dtype=torch.bfloat16, enabled=half):
            layer(Es[sl], hs[sl], xs[sl])
        if i >= warmup:
            secs.append(time.perf_counter() - t0)
    return secs, min(per_step, n)


def ref_layer_baseline(state, x, E, h, half, per_step, steps, warmup, what):
    import torch
    secs, nb = ref_layer_steps(state, x, E, h, half, per_step, steps, warmup)
    tok = nb * x.shape[1]
    return {'value': tok * len(secs) / sum(secs), 'unit': UNIT, 'cores': torch.get_num_threads(),
            'kind': 'reference', 'ms_per_step': 1e3 * statistics.median(secs),
            'sample': '%s: asrn.ASRNLayer of the reference (baseline/_ref) on the host cores, torch CPU%s, %d step(s) '
                      'of %d sequence(s) x %d tokens after %d warm-up' % (what, ', bf16 autocast' if half else '',
                                                                          len(secs), nb, x.shape[1], warmup)}


def ref_generation(prompts, B=4, steps=6, warmup=2):
    """The reference's O(1) writer (_Escritor(o1=True), asrn/nucleo.py:1717-1854) on the host cores: the
    configuration-3 model (create_model(V=50304, d=768, n_capas=12, semilla=0): the same weights as ours), batch B,
    bf16 autocast, greedy steps fed back. Returns {prompt: {step_ms, prefill_s}}."""
    import torch
    from asrn_b200 import synthetic
    asrn = import_reference()
    from asrn import nucleo
    torch.set_num_threads(host_cores())
    m = asrn.create_model(V=V, d=D, n_capas=12, semilla=0).eval()
    out = {}
    for L0 in prompts:
        x0 = torch.from_numpy(synthetic.config_tokens('cfg5', B=B, L=L0, seed=0))
        with torch.no_grad(), torch.autocast('cpu', dtype=torch.bfloat16):
            esc = nucleo._Escritor(m, True, o1=True)
            t0 = time.perf_counter()
            lg = esc.inicio(x0, L0 + steps + warmup + 2)
            pre = time.perf_counter() - t0
            nxt = lg.argmax(-1)
            secs = []
            for k in range(warmup + steps):
                t0 = time.perf_counter()
                lg = esc.paso(nxt)
                nxt = lg.argmax(-1)
                if k >= warmup:
                    secs.append(time.perf_counter() - t0)
        out[str(L0)] = {'step_ms': 1e3 * statistics.median(secs), 'prefill_s': pre}
        del esc
    return out, torch.get_num_threads()


def ref_cfg1():
    """The reference on configuration 1 (host cores, fp32): model forward on 8 x 256 bytes and generate(top_k=1) of
    200 tokens from a 512-token prompt."""
    import torch
    from asrn_b200 import synthetic
    asrn = import_reference()
    torch.set_num_threads(host_cores())
    m = asrn.create_model(V=256, d=64, n_capas=4, semilla=0).eval()
    x = torch.from_numpy(synthetic.config_tokens('cfg1', B=8, L=256, seed=0))
    x0 = torch.from_numpy(synthetic.uniform_bytes_with_repeats(1, 4096, seed=0)[:, :512])
    with torch.no_grad():
        m(x)
        secs = []
        for _ in range(3):
            t0 = time.perf_counter()
            m(x)
            secs.append(time.perf_counter() - t0)
    t0 = time.perf_counter()
    asrn.generate(m, x0, n_nuevos=200, top_k=1, devolver_logits=False)
    gen_s = time.perf_counter() - t0
    return {'forward_ms': 1e3 * statistics.median(secs), 'generate_ms_per_token': gen_s / 200 * 1e3,
            'cores': torch.get_num_threads(), 'kind': 'reference'}


# ---------------------------------------------------------------------------------------------------------------------
# main leg: configuration 3 (the headline)
# ---------------------------------------------------------------------------------------------------------------------

def dist_env():
    rank = int(os.environ.get('RANK', 0))
    world = int(os.environ.get('WORLD_SIZE', 1))
    local = int(os.environ.get('LOCAL_RANK', 0))
    return rank, world, local


def load_profile_traffic():
    """Per-token DRAM bytes of the scoring kernel from the committed ncu summary (profiles/), or None."""
    p = os.path.join(HERE, 'profiles', 'k_score_tc_cfg3_traffic.json')
    try:
        with open(p) as f:
            t = json.load(f)
        return t.get('dram_bytes_per_token')
    except (OSError, ValueError):
        return None


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    rank, world, local = dist_env()
    if world > 1:
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    from asrn_b200 import _lib, stages
    hbm, peak_src = peaks()
    out = None
    legs = {}
    if args.workload == 'cfg3':
        layer = make_layer_params().to(dev).eval()
        x_np, E_np, h_np, _table = make_inputs(args.batch, args.seq, rank)
        cpu_info = None
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            try:
                state = {k: v.detach().cpu() for k, v in layer.state_dict().items()}
                n = min(REF_CHUNK, args.batch)
                cpu_info = ref_layer_baseline(state, x_np[:n], E_np[:n], h_np[:n], True, n, 2, 1,
                                              'the headline workload')
            except Exception as exc:                              # the reference is not installed here
                cpu_info = {'unavailable': '%s: %s' % (type(exc).__name__, exc)}
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
        kern, ours_k, names = count_graph_kernels(graph) if graph is not None else (None, None, None)
        if world > 1:
            dist.barrier()
        ms, step_ms = timed(run, args.steps, clocks, barrier=True)
        if world > 1:
            dist.barrier()
        clk = clocks.stop()

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
            # replayed as a CUDA graph like the forward: an eager loop's host work (allocations, argument
            # preparation) can fall behind the 1.8 ms launches when the host cores are busy and leave gaps on the device
            srun, _, sgraph = graph_or_eager(call, args.eager)
            score_ms, _ = timed(srun, args.steps)
            score_ms /= args.steps
            del srun, sgraph, ctx, Bt, hs, orden, ids_o

        del run, graph
        torch.cuda.empty_cache()

        # end to end through the public API with pinned host buffers, copies overlapped with compute
        host_in = [torch.from_numpy(a).pin_memory() for a in (E_np, h_np, x_np)]
        host_out = torch.empty(h_np.shape, dtype=torch.float32).pin_memory()

        def fwd(Ed, hd, xd):
            with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
                return layer(Ed, hd, xd)

        e2e_ms = e2e_pipelined(fwd, host_in, host_out, dev, max(3, min(args.steps, 6)))
        del host_in, host_out, E, h, x
        torch.cuda.empty_cache()
        vals = torch.tensor([ms, e2e_ms, score_ms], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        ms, e2e_ms, score_ms = vals.tolist()
        if rank == 0:
            achieved = SCORE_BYTES_PER_TOKEN * tokens / (score_ms * 1e-3) / 1e9
            traffic_pt = load_profile_traffic()
            out = {'metric': METRIC, 'value': world * tokens * args.steps / (ms * 1e-3), 'unit': UNIT,
                   'n_gpus': world, 'steps': args.steps, 'warmup': warm, 'ms_per_step': ms / args.steps,
                   'step_ms': spread(step_ms), 'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
                   'dtype': 'bf16', 'data': 'synthetic', 'config': config(args, world),
                   'e2e': {'value': world * tokens / (e2e_ms * 1e-3), 'unit': UNIT,
                           'h2d_bytes_per_step': int(E_np.nbytes + h_np.nbytes + x_np.nbytes),
                           'd2h_bytes_per_step': int(h_np.nbytes),
                           'how': 'ASRNLayer.forward on each step\'s inputs uploaded from pinned host memory, h\' '
                                  'downloaded; uploads, forwards and downloads of consecutive steps overlap on three '
                                  'streams (two device buffer sets)'},
                   'roofline': {'bound': 'hbm', 'kernel': 'k_score_tc (candidate scoring)', 'achieved': achieved,
                                'peak': hbm, 'peak_source': peak_src, 'unit': 'GB/s', 'frac': achieved / hbm,
                                'algorithmic_bytes_per_token': SCORE_BYTES_PER_TOKEN,
                                'traffic': None if traffic_pt is None else traffic_pt * tokens,
                                'kernel_ms': score_ms,
                                'kernel_timing': 'CUDA-graph replays of the scoring call on its stream: the kernel and '
                                                 'the zero fill of its bf16 accumulator',
                                'layer_frac': LAYER_BYTES_PER_TOKEN * tokens / (ms / args.steps * 1e-3) / 1e9 / hbm},
                   'gpu_launches': (ours_k * args.steps) if ours_k else None,
                   'graph_kernels_per_step': {'all': kern, 'ours': ours_k, 'by_name': names},
                   'launch': launch_mode, 'clocks': clk,
                   'test_hooks': {'ASRN_B200_GEMM': _lib.gemm_override()}}
            if cpu_info is not None:
                out['cpu_baseline'] = cpu_info
        del layer
        torch.cuda.empty_cache()
    if args.workload == 'cfg4' or (args.workload == 'cfg3' and not args.no_legs):   # --no-legs keeps the line's own
        legs['cfg4'] = leg_cfg4(args, dev, rank, world)
    if args.workload == 'gen':
        legs['generation'] = leg_generation(args, dev, rank, world)
    if args.workload == 'model':
        legs['model'] = leg_model(args, dev, rank, world)
    if args.workload == 'localblock':
        legs['localblock'] = leg_localblock(args, dev, rank, world)
    if args.workload == 'train':
        legs['train'] = leg_train(args, dev, rank, world)
    if args.workload == 'cfg3':
        if not args.no_gen:
            legs['generation'] = leg_generation(args, dev, rank, world)
        if not args.no_legs:
            legs['cfg2'] = leg_cfg2(args, dev, rank, world)
            legs['cfg1'] = leg_cfg1(args, dev, rank, world)
            legs['model'] = leg_model(args, dev, rank, world)
            legs['train'] = leg_train(args, dev, rank, world)
    if rank == 0:
        if out is None:                       # --workload cfg4 / gen: that leg is the line
            out = dict(legs.pop({'cfg4': 'cfg4', 'gen': 'generation', 'model': 'model',
                                 'localblock': 'localblock', 'train': 'train'}[args.workload]))
        out.update({k: v for k, v in legs.items() if v is not None})
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------------------------------------------------
# legs
# ---------------------------------------------------------------------------------------------------------------------

def _max_over_ranks(vals, dev, world):
    import torch
    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def leg_cfg4(args, dev, rank, world):
    """Configuration 4: one sequence of L4 tokens, ASRNLayer(512), bf16 autocast; one GPU (graph replay) or
    sequence-sharded over the run's GPUs (asrn_b200.shard, eager: its NCCL collectives stay outside graphs). Strong
    scaling: value = tokens of the sequence per second (max-over-ranks device time)."""
    import torch
    from asrn_b200 import shard
    L = L4
    layer = make_layer_params(d=D4).to(dev).eval()
    c0, c1 = shard.chunk_bounds(L, world, rank)
    x, xc, Ec, hc, _ = make_cfg4_inputs(L, c0, c1, rank)
    xd, Ed, hd = (torch.from_numpy(a).to(dev) for a in (xc, Ec, hc))

    def step():
        with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
            if world == 1:
                return layer(Ed, hd, xd)
            return shard.forward(layer, Ed, hd, xd)

    sf = None
    if world > 1 and not args.eager:
        # the sharded forward captured as one CUDA graph per rank (NCCL collectives inside)
        with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
            sf = shard.ShardedForward(layer, Ed, hd, xd)
        # the chunk's inputs live in the graph's input buffers (copied there at construction), as with the one-GPU
        # graph replay: a step is the replay alone
        step = lambda: sf()                                # noqa: E731
    warm = warm_up(step, args.warmup, world)
    if sf is not None:
        run, mode, graph = step, 'cuda_graph', None
    else:
        run, mode, graph = graph_or_eager(step, args.eager or world > 1)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    steps = max(5, args.steps // 2)
    ms, step_ms = timed(run, steps, barrier=True)
    if sf is not None:
        torch.cuda.synchronize()
        shard.check_exchange(dev)
        exch = {k: (v.tolist() if hasattr(v, 'tolist') else v) for k, v in shard.last_exchange.items()}
        sf.close()
    del run, graph
    ms, = _max_over_ranks([ms], dev, world)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            seg = 16384             # the reference on a quarter-million-token row needs ~40 GB of host memory
            xs = x[:, :seg]
            Es = _table_rows(xs, D4, 7)
            hs = (Es + torch.randn(Es.shape, generator=torch.Generator().manual_seed(9)).numpy() * 0.5)
            state = {k: v.detach().cpu() for k, v in layer.state_dict().items()}
            cpu = ref_layer_baseline(state, xs, Es, hs.astype('float32'), True, 1, 1, 1,
                                     'the first %d tokens of the sequence' % seg)
        except Exception as exc:
            cpu = {'unavailable': '%s: %s' % (type(exc).__name__, exc)}
    del layer, xd, Ed, hd
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    hbm, src = peaks()
    step_s = ms / steps * 1e-3
    achieved = CFG4_BYTES_PER_TOKEN * (L // world) / step_s / 1e9
    leg = {'metric': METRIC, 'value': L / step_s, 'unit': UNIT, 'n_gpus': world, 'steps': steps, 'warmup': warm,
           'ms_per_step': ms / steps, 'step_ms': spread(step_ms), 'higher_is_better': True, 'scaling': 'strong',
           'dtype': 'bf16', 'data': 'synthetic', 'launch': mode,
           'config': {'workload': 'cfg4 layer: ASRNLayer(512) forward, 1 x %d tokens, bf16 autocast, fp32 E/h' % L,
                      'parallelism': ('sequence-sharded over %d GPUs, each rank one CUDA graph (NCCL all-gathers of '
                                      'the halo, clock offsets, per-position scalars, the non-empty bucket tails and '
                                      'the feature rows of the tail positions, n-gram summaries and streak maps)'
                                      % world) if world > 1 else 'single GPU'},
           'exchange': exch if world > 1 and sf is not None else None,
           'roofline': {'bound': 'hbm', 'kernel': 'whole layer forward (per GPU)', 'achieved': achieved, 'peak': hbm,
                        'peak_source': src, 'unit': 'GB/s', 'frac': achieved / hbm,
                        'algorithmic_bytes_per_token': CFG4_BYTES_PER_TOKEN}}
    if cpu is not None:
        leg['cpu_baseline'] = cpu
    return leg


def _table_rows(x, d, seed):
    import numpy as np
    table = (np.random.default_rng(seed).standard_normal((V, d)) * 0.02).astype(np.float32)
    return table[x]


def leg_cfg2(args, dev, rank, world):
    """Configuration 2: ASRNLayer(256) forward in fp32, 16 x 4096 tokens sharded over the GPUs (graph replay)."""
    import torch
    b = max(1, B2 // world)
    layer = make_layer_params(d=D2).to(dev).eval()
    x, E, h = make_cfg2_inputs(b, rank)
    xd, Ed, hd = (torch.from_numpy(a).to(dev) for a in (x, E, h))

    def step():
        with torch.no_grad():
            return layer(Ed, hd, xd)

    warm_up(step, args.warmup, world)
    run, mode, graph = graph_or_eager(step, args.eager)
    ms, step_ms = timed(run, args.steps)
    del run, graph
    ms, = _max_over_ranks([ms], dev, world)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            state = {k: v.detach().cpu() for k, v in layer.state_dict().items()}
            cpu = ref_layer_baseline(state, x[:REF_CHUNK], E[:REF_CHUNK], h[:REF_CHUNK], False, REF_CHUNK, 2, 1,
                                     'configuration 2')
        except Exception as exc:
            cpu = {'unavailable': '%s: %s' % (type(exc).__name__, exc)}
    del layer, xd, Ed, hd
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    hbm, src = peaks()
    tokens = world * b * L2
    step_s = ms / args.steps * 1e-3
    achieved = CFG2_BYTES_PER_TOKEN * b * L2 / step_s / 1e9
    leg = {'metric': METRIC, 'value': tokens / step_s, 'unit': UNIT, 'ms_per_step': ms / args.steps,
           'step_ms': spread(step_ms), 'dtype': 'f32', 'launch': mode, 'scaling': 'weak',
           'config': {'workload': 'cfg2 layer: ASRNLayer(256) forward, fp32, %d x %d tokens per GPU' % (b, L2)},
           'roofline': {'bound': 'hbm', 'kernel': 'whole layer forward (per GPU)', 'achieved': achieved, 'peak': hbm,
                        'peak_source': src, 'unit': 'GB/s', 'frac': achieved / hbm,
                        'algorithmic_bytes_per_token': CFG2_BYTES_PER_TOKEN}}
    if cpu is not None:
        leg['cpu_baseline'] = cpu
    return leg


def ref_train_baseline(state, x, E, h, G, steps=2, warmup=1):
    """The reference's ASRNLayer forward + backward of sum(h' * G) on the host cores (torch CPU, bf16 autocast), one
    sequence per step: tokens/s."""
    import torch
    asrn = import_reference()
    torch.set_num_threads(host_cores())
    layer = asrn.ASRNLayer(E.shape[-1])
    layer.load_state_dict(state)
    layer.train()
    xs, Gs = torch.from_numpy(x), torch.from_numpy(G)
    secs = []
    for i in range(warmup + steps):
        Es = torch.from_numpy(E).requires_grad_()
        hs = torch.from_numpy(h).requires_grad_()
        t0 = time.perf_counter()
        with torch.autocast('cpu', dtype=torch.bfloat16):
            y = layer(Es, hs, xs)
        (y.float() * Gs).sum().backward()
        if i >= warmup:
            secs.append(time.perf_counter() - t0)
        layer.zero_grad(set_to_none=True)
    tok = x.shape[0] * x.shape[1]
    return {'value': tok * len(secs) / sum(secs), 'unit': 'tokens/s', 'cores': torch.get_num_threads(),
            'kind': 'reference', 'ms_per_step': 1e3 * statistics.median(secs),
            'sample': 'asrn.ASRNLayer of the reference (baseline/_ref), forward + backward on the host cores, torch '
                      'CPU, bf16 autocast, %d step(s) of %d x %d tokens after %d warm-up' % (len(secs), x.shape[0],
                                                                                            x.shape[1], warmup)}


def leg_train(args, dev, rank, world):
    """Training step of the layer on one GPU (rank 0; the other ranks skip it): ASRNLayer(768) in training mode, bf16
    autocast, forward + backward of sum(h' * G) on TRAIN_B x 8192 tokens (cfg3 shapes): the differentiable path with
    the bucket attention and the scans on the training kernels. Eager (the backward is autograd's)."""
    import numpy as np
    import torch
    if rank != 0:
        return None
    layer = make_layer_params(d=D).to(dev).train()
    x, E, h, _ = make_inputs(TRAIN_B, L_SEQ, 0)
    G = np.random.default_rng(5).standard_normal(E.shape).astype(np.float32)
    xd, Ed, hd, Gd = (torch.from_numpy(a).to(dev) for a in (x, E, h, G))
    Ed.requires_grad_()
    hd.requires_grad_()

    def step():
        with torch.autocast('cuda', dtype=torch.bfloat16):
            y = layer(Ed, hd, xd)
        (y.float() * Gd).sum().backward()
        layer.zero_grad(set_to_none=True)
        Ed.grad = None
        hd.grad = None

    warm_up(step, args.warmup, 1)
    n = max(3, args.steps // 4)
    ms, step_ms = timed(step, n)
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        try:
            state = {k: v.detach().cpu() for k, v in layer.state_dict().items()}
            seg = 2048
            cpu = ref_train_baseline(state, x[:1, :seg], E[:1, :seg], h[:1, :seg], G[:1, :seg])
        except Exception as exc:
            cpu = {'unavailable': '%s: %s' % (type(exc).__name__, exc)}
    del layer, xd, Ed, hd, Gd
    torch.cuda.empty_cache()
    step_s = ms / n * 1e-3
    leg = {'metric': 'asrn_layer_train_tokens_per_s', 'value': TRAIN_B * L_SEQ / step_s, 'unit': 'tokens/s',
           'ms_per_step': ms / n, 'step_ms': spread(step_ms), 'dtype': 'bf16', 'launch': 'eager',
           'config': {'workload': 'ASRNLayer(768) forward + backward of sum(h\' * G), training mode, bf16 autocast, '
                                  '%d x %d tokens (cfg3 shapes)' % (TRAIN_B, L_SEQ)}}
    if cpu is not None:
        leg['cpu_baseline'] = cpu
    return leg


def leg_cfg1(args, dev, rank, world):
    """Configuration 1 on one GPU (rank 0; the other ranks skip it): create_model(V=256, d=64, n_capas=4, semilla=0)
    forward on 8 x 256 bytes (fp32, graph replay), then generate(top_k=1) of 200 tokens from a 512-token prompt end to
    end through the public API."""
    import torch
    import asrn_b200
    from asrn_b200 import synthetic
    vals = [0.0, 0.0]
    if rank == 0:
        m = asrn_b200.create_model(V=256, d=64, n_capas=4, semilla=0).to(dev).eval()
        x = torch.from_numpy(synthetic.config_tokens('cfg1', B=8, L=256, seed=0)).to(dev)
        x0 = torch.from_numpy(synthetic.uniform_bytes_with_repeats(1, 4096, seed=0)[:, :512])

        def step():
            with torch.no_grad():
                return m(x)

        warm_up(step, args.warmup, 1)
        run, mode, graph = graph_or_eager(step, args.eager)
        ms, _ = timed(run, args.steps)
        del run, graph
        asrn_b200.generate(m, x0, n_nuevos=8, top_k=1, devolver_logits=False)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        asrn_b200.generate(m, x0, n_nuevos=200, top_k=1, devolver_logits=False)
        torch.cuda.synchronize()
        vals = [ms / args.steps, (time.perf_counter() - t0) / 200 * 1e3]
        del m
        torch.cuda.empty_cache()
    if rank != 0:
        return None
    leg = {'forward_ms': vals[0], 'forward_tokens_per_s': 8 * 256 / (vals[0] * 1e-3),
           'generate_ms_per_token': vals[1], 'dtype': 'f32', 'launch': mode,
           'config': {'workload': 'cfg1: create_model(V=256, d=64, n_capas=4, semilla=0); forward on 8 x 256 '
                                  'bytes with 30 % planted repeats; generate(top_k=1) of 200 tokens from a 512-token '
                                  'prompt (host tokens in and out)'}}
    if not args.no_cpu_baseline:
        try:
            leg['cpu_baseline'] = ref_cfg1()
        except Exception as exc:
            leg['cpu_baseline'] = {'unavailable': '%s: %s' % (type(exc).__name__, exc)}
    return leg


MODEL_B = 4


def leg_model(args, dev, rank, world):
    """The cfg3 model forward on one GPU (rank 0; the other ranks skip it): create_model(V=50304, d=768, n_capas=12)
    (6 ASRN layers, 12 local blocks, tied head) random init, MODEL_B x 8192 Zipf+repeat tokens, bf16 autocast, the
    whole forward replayed as one CUDA graph. Also timed: each ASRN layer sorting the n-grams itself, and the local
    blocks as PyTorch ops, to show what the shared sort and the fused blocks save."""
    import torch
    import asrn_b200
    from asrn_b200 import synthetic
    from asrn_b200.model import BloqueLocal
    vals = [0.0, 0.0, 0.0]
    mode = None
    if rank == 0:
        m = asrn_b200.create_model(V=V, d=D, n_capas=12, semilla=0).to(dev).eval()
        x = torch.from_numpy(synthetic.config_tokens('cfg3', B=MODEL_B, L=L_SEQ, seed=0)).to(dev)

        def step():
            with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
                return m(x)

        fused_ok = BloqueLocal._fused_ok
        for i, (shared, fused) in enumerate(((True, True), (False, True), (True, False))):
            m._ngram_shared = (lambda ok: (lambda: ok))(shared)        # sort once, or in every layer
            BloqueLocal._fused_ok = fused_ok if fused else (lambda self, h: False)
            try:
                warm_up(step, args.warmup, 1)
                run, mode_i, graph = graph_or_eager(step, args.eager)
                n = max(3, args.steps // 4)
                ms, _ = timed(run, n)
                vals[i] = ms / n
                mode = mode or mode_i
                del run, graph
            finally:
                BloqueLocal._fused_ok = fused_ok
        del m
        torch.cuda.empty_cache()
    if rank != 0:
        return None
    tokens = MODEL_B * L_SEQ
    return {'metric': 'model_fwd_tokens_per_s', 'value': tokens / (vals[0] * 1e-3), 'unit': 'tokens/s',
            'forward_ms': vals[0], 'forward_ms_sorting_in_every_layer': vals[1],
            'forward_ms_pytorch_local_blocks': vals[2], 'dtype': 'bf16', 'launch': mode,
            'config': {'workload': 'cfg3 model: create_model(V=50304, d=768, n_capas=12) random init, forward on '
                                   '%d x %d Zipf+repeat tokens, bf16 autocast (logits included)' % (MODEL_B, L_SEQ),
                       'ngram_sort': 'once per forward, shared by the 6 ASRN layers',
                       'local_blocks': 'fused (asrn_local_block: LN kernel + three tcgen05 GEMMs)'}}


LB_B = 8
LB_BYTES_PER_TOKEN = 4 * 768 * 6 + 2 * 768 * 4 + 2 * 1536 * 2      # fp32 stream 4 reads + 2 writes, bf16 z/u, f


def leg_localblock(args, dev, rank, world):
    """One cfg3 local block (BloqueLocal(768), k = 4, ff = 1536) on LB_B x 8192 tokens under bf16 autocast, fused
    (asrn_local_block) and as PyTorch ops; roofline on the fused block's HBM bytes (the fp32 residual stream read four
    times and written twice, the bf16 z / u / f intermediates written and read once)."""
    import torch
    from asrn_b200.model import BloqueLocal
    torch.manual_seed(0)
    blq = BloqueLocal(D, 4, 2 * D).to(dev).eval()
    h = torch.randn(LB_B, L_SEQ, D, device=dev)
    res = []

    def step():
        with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16):
            return blq(h)

    fused_ok = BloqueLocal._fused_ok
    for fused in (True, False):
        BloqueLocal._fused_ok = fused_ok if fused else (lambda self, x: False)
        try:
            warm_up(step, args.warmup, 1)
            run, mode, graph = graph_or_eager(step, args.eager)
            ms, _ = timed(run, args.steps)
            res.append(ms / args.steps)
            del run, graph
        finally:
            BloqueLocal._fused_ok = fused_ok
    if rank != 0:
        return None
    hbm, src = peaks()
    tokens = LB_B * L_SEQ
    achieved = LB_BYTES_PER_TOKEN * tokens / (res[0] * 1e-3) / 1e9
    return {'metric': 'local_block_tokens_per_s', 'value': tokens / (res[0] * 1e-3), 'unit': 'tokens/s',
            'ms_per_step': res[0], 'pytorch_ms_per_step': res[1], 'dtype': 'bf16', 'launch': mode,
            'config': {'workload': 'BloqueLocal(768, k=4, ff=1536), %d x %d tokens, bf16 autocast' % (LB_B, L_SEQ)},
            'roofline': {'bound': 'hbm', 'achieved': achieved, 'peak': hbm, 'peak_source': src, 'unit': 'GB/s',
                         'frac': achieved / hbm, 'algorithmic_bytes_per_token': LB_BYTES_PER_TOKEN}}


def leg_generation(args, dev, rank, world):
    """Generation leg: per prompt length, the prompt pass (prefill) then args.gen_steps greedy steps of the O(1)
    writer, each step the CUDA-graph replay of the model's step plus a device argmax feeding the next token (no host
    sync), timed with CUDA events; then the public API (generate, top_k=1) end to end at the shortest prompt; then the
    reference's writer on the host cores."""
    import torch
    import asrn_b200
    from asrn_b200 import synthetic
    from asrn_b200.writer import argmax_rows
    B = max(1, GEN_B // world)
    torch.manual_seed(0)
    m = asrn_b200.create_model(V=V, d=D, n_capas=12, semilla=0).to(dev).eval()
    prompts = sorted(set([p for p in GEN_FLAT if p < args.gen_prompt] + [args.gen_prompt]))
    res = {}
    for L0 in prompts:
        x0 = torch.from_numpy(synthetic.config_tokens('cfg5', B=B, L=L0, seed=rank)).to(dev)
        with torch.autocast('cuda', dtype=torch.bfloat16):
            w = asrn_b200.Writer(m)
            torch.cuda.synchronize()
            p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            p0.record()
            lg = w.inicio(x0, capacidad=L0 + args.gen_steps + 8)
            p1.record()
            nxt = argmax_rows(lg)
            for _ in range(3):
                nxt = argmax_rows(w.paso(nxt, copiar=False))
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.nvtx.range_push('gen_steps')          # lets a profiler select the timed steps' kernels
            e0.record()
            for _ in range(args.gen_steps):
                nxt = argmax_rows(w.paso(nxt, copiar=False))
            e1.record()
            torch.cuda.nvtx.range_pop()
            torch.cuda.synchronize()
            status = w.status()
            if any(status):
                raise RuntimeError(f'generation step status {status}')
            res[L0] = [e0.elapsed_time(e1) / args.gen_steps * 1e3, B * L0 / (p0.elapsed_time(p1) * 1e-3)]
            w.cerrar()
            del w, lg, nxt, x0
        torch.cuda.empty_cache()
    # public API end to end (host tokens in, host tokens out, sampling as the reference's): per-token cost from pairs
    # of calls that differ only in the number of new tokens (a call's fixed cost -- the prompt pass, the quote index of
    # the prompt built on the host, the step's graph capture -- varies by tens of ms, so the pairs differ by 128 tokens
    # and the median of three is taken); greedy (top_k=1) and the API's default sampling (temperature 0.8, top_k 40),
    # both drawn on the device from the reference's seeded generator stream
    L0 = prompts[0]
    x0 = torch.from_numpy(synthetic.config_tokens('cfg5', B=B, L=L0, seed=rank))
    n_a, n_b = 8, 136
    e2e_by_mode = {}
    with torch.autocast('cuda', dtype=torch.bfloat16):
        for mode, kw in (('greedy', dict(top_k=1)), ('sampled', dict(temperatura=0.8, top_k=40))):
            asrn_b200.generate(m, x0, n_nuevos=n_b, devolver_logits=False, **kw)
            per = []
            for _ in range(3):
                times = []
                for n in (n_a, n_b):
                    torch.cuda.synchronize()
                    t0 = time.perf_counter()
                    asrn_b200.generate(m, x0, n_nuevos=n, devolver_logits=False, **kw)
                    torch.cuda.synchronize()
                    times.append(time.perf_counter() - t0)
                per.append((times[1] - times[0]) / (n_b - n_a) * 1e6)
            e2e_by_mode[mode] = statistics.median(per)
    e2e_us = e2e_by_mode['greedy']
    del m
    torch.cuda.empty_cache()
    flat = [res[p][0] for p in prompts]
    vals = _max_over_ranks(flat + [e2e_us, e2e_by_mode['sampled']], dev, world)
    step_us = dict(zip(prompts, vals[:len(prompts)]))
    e2e_us, e2e_sampled_us = vals[-2], vals[-1]
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            ps = [int(p) for p in args.gen_cpu_prompts.split(',') if p]
            ref, cores = ref_generation(ps)
            cpu = {'value': statistics.median([r['step_ms'] for r in ref.values()]) * 1e3, 'unit': 'us/token',
                   'cores': cores, 'kind': 'reference', 'step_us_by_prompt': {k: r['step_ms'] * 1e3
                                                                               for k, r in ref.items()},
                   'prefill_s_by_prompt': {k: r['prefill_s'] for k, r in ref.items()},
                   'sample': "the reference's _Escritor(o1=True) (baseline/_ref) on the host cores, torch CPU, bf16 "
                             "autocast, batch 4 (a step writes one token of each of the 4 sequences), the same "
                             "model weights and prompt generator, greedy steps fed back"}
        except Exception as exc:
            cpu = {'unavailable': '%s: %s' % (type(exc).__name__, exc)}
    if rank != 0:
        return None
    main = step_us[args.gen_prompt]
    leg = {'metric': 'gen_us_per_token', 'value': main, 'unit': 'us/token', 'higher_is_better': False,
           'workload': 'cfg5: create_model(V=50304, d=768, n_capas=12) random init, %d sequences (%d per GPU), '
                       'Zipf+repeat prompts of %d tokens, %d greedy steps (CUDA-graph step + device argmax), bf16 '
                       'autocast' % (B * world, B, args.gen_prompt, args.gen_steps),
           'step_us_by_prompt': {str(k): v for k, v in step_us.items()},
           'prefill_tokens_per_s_by_prompt': {str(k): res[k][1] * world for k in prompts},
           'tokens_per_s': B * world / (main * 1e-6),
           'e2e': {'value': e2e_us, 'unit': 'us/token',
                   'sampled_us_per_token': e2e_sampled_us,
                   'api': 'asrn_b200.generate(top_k=1, devolver_logits=False), host prompt of %d tokens; per-token '
                          'cost = difference of a %d- and an %d-token call / %d, median of 3 pairs; '
                          'sampled_us_per_token: the same with '
                          'temperatura=0.8, top_k=40 (the API default); draws on the device from the reference\'s '
                          'seeded CPU generator stream' % (L0, n_b, n_a, n_b - n_a)}}
    if cpu is not None:
        leg['cpu_baseline'] = cpu
    return leg


# ---------------------------------------------------------------------------------------------------------------------
# --impl reference
# ---------------------------------------------------------------------------------------------------------------------

def run_reference(args):
    """The reference's own CPU implementation of the headline workload, on rank 0 (other ranks exit without work):
    asrn.ASRNLayer from baseline/_ref, torch on the host cores, bf16 autocast, REF_CHUNK sequences per step."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    try:
        import_reference()
    except Exception as exc:
        print(json.dumps({'impl': 'reference', 'unavailable': 'the reference is not installed in baseline/_ref (%s)'
                          % exc}), flush=True)
        return 0
    import torch
    layer = make_layer_params()
    state = {k: v.detach() for k, v in layer.state_dict().items()}
    n = max(REF_CHUNK, min(2 * REF_CHUNK, args.batch))
    x, E, h, _ = make_inputs(n, args.seq, 0)
    steps = max(1, min(args.steps, 12))
    secs, nb = ref_layer_steps(state, x, E, h, True, REF_CHUNK, steps, max(1, min(args.warmup, 2)))
    tok = nb * args.seq
    v = tok * len(secs) / sum(secs)
    info = {'value': v, 'unit': UNIT, 'cores': torch.get_num_threads(), 'kind': 'reference',
            'sample': 'asrn.ASRNLayer of the reference (baseline/_ref), torch CPU on the host cores, bf16 autocast: '
                      '%d steps of %d sequences x %d tokens of the headline workload (the same weights and input '
                      'generator)' % (len(secs), nb, args.seq)}
    out = {'metric': METRIC, 'value': v, 'unit': UNIT, 'n_gpus': world, 'steps': len(secs), 'warmup': args.warmup,
           'ms_per_step': 1e3 * sum(secs) / len(secs), 'higher_is_better': True, 'scaling': 'weak',
           'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic', 'impl': 'reference', 'config': config(args, world),
           'cpu_baseline': info,
           'e2e': {'value': v, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    if not args.no_gen:
        try:
            ref, cores = ref_generation([int(p) for p in args.gen_cpu_prompts.split(',') if p])
            out['generation'] = {'metric': 'gen_us_per_token', 'unit': 'us/token', 'higher_is_better': False,
                                 'value': statistics.median([r['step_ms'] for r in ref.values()]) * 1e3,
                                 'step_us_by_prompt': {k: r['step_ms'] * 1e3 for k, r in ref.items()},
                                 'cores': cores, 'workload': "_Escritor(o1=True), batch 4, bf16 autocast, host cores"}
        except Exception as exc:
            out['generation'] = {'unavailable': '%s: %s' % (type(exc).__name__, exc)}
    print(json.dumps(out), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == 'reference':
        return run_reference(args)
    return run_ours(args)


if __name__ == '__main__':
    sys.exit(main())
