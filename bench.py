"""Benchmark: PI0 batch-1 action-chunk latency and chunks/s on B200.

    python bench.py [--gpus N --steps K --warmup W] [--impl b200|reference]
                    [--workload pi0|pi05|loop]

A "step" is one action chunk: one full PI0 inference (config[2]: 3 views
224x224 uint8 -> SigLIP So400m -> Gemma-2B prefix prefill over 816 rows
writing the bf16 KV cache -> 10 Euler steps of the 18-layer action expert
over 51 suffix tokens), i.e. one replay of the engine's CUDA graph.
Weights are seeded random bf16 of the real architecture (no checkpoint is
available); inputs are seeded synthetic tensors of the benchmark's shapes.
Every chunk streams ~6.6 GB of weights, far more than the 126 MB L2, so no L2
flush is needed between timed iterations.

N > 1 (torchrun): one independent replica per GPU (the path has no
intra-request shard, so there is no collective on the data path); the
barrier and the max-over-ranks reduction of the timings use NCCL.
`value` = N * 1000 / (max-over-ranks ms per chunk).

--impl reference times the reference algorithm's CPU path (the fp32 oracle
port of the eager modules, all host threads) on a bounded sample and prints
the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = ('PI0 batch-1 action-chunk latency (ms) and chunks/s at 1/2/4/8 '
          'B200; roofline %')
PEAKS_FALLBACK = {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0,
                  'bf16_tflops_sustained': 1400.0}


def load_peaks():
    p = os.path.join(ROOT, 'MEASURED_PEAKS.json')
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), 'measured'
    return PEAKS_FALLBACK, 'fallback'


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    Q = ('index,clocks.sm,clocks.max.sm,power.draw,'
         'clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
         'clocks_event_reasons.hw_thermal_slowdown,'
         'clocks_event_reasons.sw_thermal_slowdown,'
         'clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.lines = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ['nvidia-smi', f'--query-gpu={self.Q}',
                 '--format=csv,noheader,nounits', '-i', str(self.idx),
                 '-lms', '200'], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {'sm_mhz': None, 'sm_max_mhz': None,
                    'reasons': ['unsampled']}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown',
                 'sw_power_cap']
        for ln in self.lines:
            f = [x.strip() for x in ln.split(',')]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == 'active':
                    reasons.add(n)
        return {'sm_mhz': statistics.median(sm) if sm else None,
                'sm_max_mhz': mx, 'reasons': sorted(reasons),
                'samples': len(sm)}


# ---------------------------------------------------------------------------
# CPU reference arm (oracle port of the eager reference, all host threads)
# ---------------------------------------------------------------------------

def _reference_or_none():
    """The reference's own eager modules (oracle/ref_shim.py, loaded from
    baseline/_ref or $FLUXVLA_REF), or None when not installed."""
    try:
        from oracle import ref_shim
        if ref_shim.reference_root() is None:
            return None, None
        return ref_shim, ref_shim.load_reference()
    except Exception as e:  # noqa: BLE001
        print(f'# reference modules unavailable: {e}', file=sys.stderr)
        return None, None


def _chunk_inputs(cfg, n_tok, seed=1):
    g = torch.Generator().manual_seed(seed)
    u8 = torch.randint(0, 256, (cfg.n_views, 224, 224, 3), generator=g,
                       dtype=torch.uint8)
    toks = torch.randint(0, cfg.vocab, (1, n_tok), generator=g)
    state = torch.randn(1, cfg.state_dim, generator=g)
    noise = torch.randn(1, cfg.n_actions, cfg.action_dim, generator=g)
    return u8, toks, state, noise


class CpuChunk:
    """One whole action chunk of the workload on the host cores, fp32: the
    reference's own eager PI0FlowMatching / PI05FlowMatching
    .predict_action when the reference is installed ('reference'), else the
    oracle port of the same algorithm ('port').  Images are normalised as
    the reference's NormalizeImages transform does, outside the timed call
    for the reference (its transform runs before predict_action)."""

    def __init__(self, workload: str, threads: int):
        from fluxvla_b200.config import PI0Config, pi05_config
        from fluxvla_b200.weights import make_weights
        torch.set_num_threads(threads)
        self.threads = threads
        pi05 = workload == 'pi05'
        self.cfg = cfg = pi05_config() if pi05 else PI0Config()
        self.n_tok = 80 if pi05 else 48
        t0 = time.perf_counter()
        W = make_weights(cfg, seed=0)
        shim, ref = _reference_or_none()
        self.kind = 'port' if ref is None else 'reference'
        u8, self.toks, self.state, self.noise = _chunk_inputs(cfg,
                                                              self.n_tok)
        self.u8 = u8
        V = cfg.n_views
        mean = torch.tensor(cfg.img_mean)[:, None, None]
        std = torch.tensor(cfg.img_std)[:, None, None]
        self.pix = ((u8.float().permute(0, 3, 1, 2) - mean) /
                    (std + 1e-8)).reshape(1, 3 * V, 224, 224)
        if ref is not None:
            with shim.no_param_init():
                self.model = shim.build_ref_model(ref, cfg)
            shim.load_weights(self.model, cfg, W)
            del W
        else:
            self.W = {k: v.float() for k, v in W.items()}
        self.setup_s = time.perf_counter() - t0

    @torch.no_grad()
    def __call__(self):
        if self.kind == 'reference':
            return self.model.predict_action(
                self.pix, self.toks, self.state,
                img_masks=torch.ones(1, self.cfg.n_views, dtype=torch.bool),
                lang_masks=torch.ones(1, self.n_tok, dtype=torch.bool),
                noise=self.noise.clone())
        from oracle import pi0_oracle as O
        return O.predict_action(self.cfg, self.W, self.u8, self.toks,
                                self.state, self.noise)

    def sample_doc(self):
        who = ('the reference\'s own eager {} .predict_action (fp32, loaded '
               'unmodified from baseline/_ref through oracle/ref_shim.py)'
               if self.kind == 'reference' else
               'the fp32 oracle port of the eager {} path')
        name = 'PI05FlowMatching' if self.cfg.adarms else 'PI0FlowMatching'
        return (f'one whole config chunk per step: {who.format(name)}, '
                f'{self.threads} host threads')


def time_cpu_chunks(chunk: CpuChunk, n: int, warmup: int = 1):
    for _ in range(warmup):
        chunk()
    ts = []
    for _ in range(n):
        t0 = time.perf_counter()
        chunk()
        ts.append(time.perf_counter() - t0)
    return ts


def cpu_layer0_sample():
    """config[0] on the host: the reference's own ConditionGemmaModel layer
    (or the oracle port) over x [1,816,2048] fp32, causal, one warm-up and
    three timed runs.  -> (ms, kind, cores, sample)."""
    from fluxvla_b200.config import PI0Config
    from fluxvla_b200.weights import make_weights
    from oracle import pi0_oracle as O
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = PI0Config(llm_layers=1)
    W = make_weights(cfg, 0, parts=('llm',))
    del W['llm.embed']
    x = torch.randn(1, 816, cfg.llm_width,
                    generator=torch.Generator().manual_seed(1))
    shim, ref = _reference_or_none()
    if ref is not None:
        g = ref.cg.ConditionGemmaModel(**{
            k: v for k, v in shim._gemma_cfg(cfg.llm_width, cfg.llm_mlp, 1,
                                             cfg, False).items()
            if k != 'type'}).float().eval()
        g.config._attn_implementation = 'eager'
        sd = {theirs[len('llm_backbone.'):]: W[ours].float()
              for ours, theirs in shim.name_map(cfg).items() if ours in W}
        g.load_state_dict(sd, strict=False)
        layer = g.layers[0]
        pos = torch.arange(816)[None]
        pe = g.rotary_emb(x, pos)
        causal = torch.full((816, 816), torch.finfo(torch.float32).min
                            ).triu(1)[None, None]

        def f():
            return layer(x, attention_mask=causal, position_ids=pos,
                         position_embeddings=pe)[0]
        kind = 'reference'
    else:
        Wf = {k: v.float() for k, v in W.items()}

        def f():
            return O.gemma_layer_causal(cfg, Wf, x)
        kind = 'port'
    with torch.no_grad():
        f()
        ts = []
        for _ in range(3):
            t0 = time.perf_counter()
            f()
            ts.append(time.perf_counter() - t0)
    ms = statistics.median(ts) * 1e3
    return ms, kind, threads, (f'median of 3 forwards of one {kind} Gemma-2B '
                               f'layer (fp32, {threads} threads)')


def workload_name(w):
    return {
        'pi0': 'config[2]: PI0 batch-1 full inference, 3 views 224x224 uint8, '
               '48 prompt tokens, 816-row prefix, state + 50 action tokens, '
               '10 Euler steps',
        'pi05': 'config[3]: PI0.5 batch-1 full inference, 3 views, 80 prompt '
                'tokens (48 text + 32 state), 848-row prefix, 50 action '
                'tokens, adaRMS expert, 10 Euler steps',
        'loop': 'config[1]: PI0 action-expert loop only, 816-row prefix KV '
                'cache, 51 suffix tokens, 10 Euler steps',
        'layer0': 'config[0]: one Gemma-2B decoder layer, x [1,816,2048] '
                  'f32 ~N(0,1), causal mask, positions 0..815',
    }[w]


def run_reference(args):
    """The reference's CPU path, timed: whole chunks of the workload (pi0 /
    pi05 / loop use the full PI0 or PI0.5 predict_action) or config[0]
    layers.  The number of timed chunks is capped at 5 after one warm-up
    (a chunk takes seconds on the host); ``steps`` reports what was timed."""
    if int(os.environ.get('RANK', '0')) != 0:
        return 0
    threads = os.cpu_count() or 1
    if args.workload == 'layer0':
        ms, kind, cores, sample = cpu_layer0_sample()
        v, unit, n = 1000.0 / ms, 'layers/s', 3
    else:
        chunk = CpuChunk('pi05' if args.workload == 'pi05' else 'pi0',
                         threads)
        n = max(1, min(args.steps, 5))
        ts = time_cpu_chunks(chunk, n, warmup=1)
        ms = statistics.median(ts) * 1e3
        v, unit, kind, cores = 1000.0 / ms, 'chunks/s', chunk.kind, threads
        sample = chunk.sample_doc() + (
            f'; median of {n} timed chunks after 1 warm-up '
            f'(setup {chunk.setup_s:.0f} s untimed)')
    line = {'metric': METRIC, 'value': v, 'unit': unit,
            'n_gpus': args.gpus, 'steps': n, 'warmup': 1,
            'ms_per_step': ms, 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
            'impl': 'reference',
            'config': {'workload': workload_name(args.workload),
                       'parallelism': 'one host process (rank 0)'},
            'cpu_baseline': {'value': v, 'unit': unit, 'cores': cores,
                             'kind': kind, 'sample': sample},
            'e2e': {'value': v, 'unit': unit, 'h2d_bytes_per_step': 0,
                    'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------

def captured_traffic():
    """(bytes, note) of the expert step's DRAM traffic per launch from the
    line ``traffic_bytes: N source_sha256: H`` of
    profiles/expert_step_kernel.md, when H is the sha256 of the kernel
    source (csrc/expert_mega.cuh) now; else (None, reason)."""
    import hashlib
    import re
    src = os.path.join(ROOT, 'fluxvla_b200', 'csrc', 'expert_mega.cuh')
    prof = os.path.join(ROOT, 'profiles', 'expert_step_kernel.md')
    try:
        with open(src, 'rb') as f:
            sha = hashlib.sha256(f.read()).hexdigest()
        with open(prof) as f:
            m = re.search(r'traffic_bytes: (\d+) source_sha256: ([0-9a-f]{64})',
                          f.read())
    except OSError:
        return None, 'no capture'
    if not m:
        return None, 'no capture'
    if m.group(2) != sha:
        return None, 'capture is of another kernel source (stale)'
    return float(m.group(1)), f'ncu capture of source sha256 {sha[:12]}'


def run_b200(args):
    import torch.distributed as dist

    from fluxvla_b200 import ops
    from fluxvla_b200._lib import EPI_GEGLU
    from fluxvla_b200.config import PI0Config, pi05_config
    from fluxvla_b200.engine import PI0EngineB200
    from fluxvla_b200.weights import make_weights

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    dev = torch.device('cuda', local)
    if world > 1:
        dist.init_process_group('nccl', device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    w = args.workload
    if w == 'layer0':
        return run_layer0(args, world, rank, local, dev, barrier,
                          max_over_ranks)
    depth = {} if not args.depth else dict(
        vis_layers=args.depth, llm_layers=args.depth, exp_layers=args.depth,
        vocab=4096)
    cfg = pi05_config(**depth) if w == 'pi05' else PI0Config(**depth)
    n_tok = 80 if w == 'pi05' else 48
    E = cfg.n_views * cfg.tokens_per_view + n_tok
    parts = ('exp', 'heads') if w == 'loop' else ('vision', 'llm', 'exp',
                                                  'heads')
    W = make_weights(cfg, seed=0, parts=parts, device=dev)
    eng = PI0EngineB200(cfg, W, prefix_len=E, device=dev)
    del W
    torch.cuda.empty_cache()

    if w == 'serve':
        return run_serve(args, cfg, eng, n_tok, E, world, rank, local, dev)

    g = torch.Generator().manual_seed(1 + rank)
    imgs = torch.randint(0, 256, (cfg.n_views, 224, 224, 3), generator=g,
                         dtype=torch.uint8).pin_memory()
    toks = torch.randint(0, cfg.vocab, (1, n_tok), generator=g).pin_memory()
    state = torch.randn(1, cfg.state_dim, generator=g).pin_memory()
    noise = torch.randn(1, cfg.n_actions, cfg.action_dim,
                        generator=g).pin_memory()
    if w == 'loop':
        kc = torch.randn(cfg.exp_layers, E, cfg.head_dim, generator=g)
        vc = torch.randn(cfg.exp_layers, E, cfg.head_dim, generator=g)
        eng.set_prefix_cache(kc.to(dev, torch.bfloat16),
                             vc.to(dev, torch.bfloat16))

        def call():
            eng.load_inputs(state=state, noise=noise)
            if eng.graph is None:
                eng.capture(prefix=False)
            eng.replay()
            return eng.actions.to('cpu')
        h2d = state.numel() * 4 + noise.numel() * 4
    else:
        def call():
            return eng.predict_action(imgs, toks, state, noise=noise)
        h2d = (imgs.numel() + toks.numel() * 8 + state.numel() * 4 +
               noise.numel() * 4 + E * (1 + 4) + eng.S * 4)
    d2h = cfg.n_actions * cfg.action_dim * 4

    call()  # capture + first run
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        eng.replay()
    torch.cuda.synchronize(dev)
    if args.profile:
        # one graph replay bracketed for `ncu --profile-from-start off`
        torch.cuda.cudart().cudaProfilerStart()
        eng.replay()
        torch.cuda.synchronize(dev)
        torch.cuda.cudart().cudaProfilerStop()
        print(json.dumps({'profiled_launches': eng.launches_per_call}))
        return 0

    # ---- device-timed region: K graph replays (inputs resident) ----
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.6)
    barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        eng.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)

    # ---- end-to-end through predict_action (pinned H2D + D2H per chunk) --
    barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = call()
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3 / args.steps)
    barrier()
    assert torch.isfinite(out).all()

    # ---- roofline: the dominant kernel (the persistent expert step, one
    # launch per denoise step) timed alone with CUDA events on its stream;
    # algorithmic bytes per launch = expert weights + prefix K/V of all layers
    peaks, peak_kind = load_peaks()
    L = cfg.exp_layers
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    xargs = eng._expert_args(0)
    saved = eng.B['e_res'].clone()
    reps = 20
    ev[0].record(stream)
    for _ in range(reps):
        ops.expert_step(xargs)
    ev[1].record(stream)
    torch.cuda.synchronize(dev)
    eng.B['e_res'].copy_(saved)
    t_launch = ev[0].elapsed_time(ev[1]) / reps * 1e-3
    wbytes = sum(eng.P[f'exp.{n}_all'].numel() * 2
                 for n in ('qkv', 'o_w', 'gu', 'down_w'))
    kvbytes = 2 * L * E * cfg.head_dim * 2
    ach = (wbytes + kvbytes) / t_launch / 1e9
    # DRAM bytes (read + write) of one launch from the committed ncu
    # capture, used only while the kernel source is the one captured
    traffic, traffic_src = captured_traffic() if (
        L == 18 and E == 816 and not args.depth) else (None, None)
    roof = {'kernel': f'fvb::mega::expert_step_kernel ({L} expert layers of one '
                      'denoise step, persistent, 148 CTAs)',
            'bound': 'hbm', 'achieved': ach, 'peak': peaks['hbm_gbs'],
            'unit': 'GB/s', 'frac': ach / peaks['hbm_gbs'],
            'peak_source': f'{peak_kind} HBM copy (kernel timed alone)',
            'traffic': traffic, 'traffic_source': traffic_src,
            'launch_us': t_launch * 1e6,
            'algorithmic_bytes_per_launch': wbytes + kvbytes}
    roof_prefill = None
    if w != 'loop':
        P, B = eng.P, eng.B
        reps, Lp = 3, cfg.llm_layers - 1
        ev[0].record(stream)
        for _ in range(reps):
            for i in range(Lp):
                ops.gemm(B['l_xn'], P[f'llm.l{i}.gu'], B['l_h'],
                         epilogue=EPI_GEGLU, block_n=256)
        ev[1].record(stream)
        torch.cuda.synchronize(dev)
        t_g = ev[0].elapsed_time(ev[1]) / (reps * Lp) * 1e-3
        flops = 2.0 * E * cfg.llm_width * 2 * cfg.llm_mlp
        roof_prefill = {
            'kernel': 'gemm_tc_kernel<256,4,GEGLU> Gemma-2B gate/up '
                      f'[{E}x2048]x[32768x2048]^T', 'bound': 'tensor',
            'achieved': flops / t_g / 1e12, 'peak': peaks['bf16_tflops'],
            'unit': 'TFLOP/s', 'frac': flops / t_g / 1e12 / peaks['bf16_tflops'],
            'peak_source': f'{peak_kind} burst bf16 (kernel timed alone)',
            'launch_us': t_g * 1e6}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        chunk = CpuChunk('pi05' if w == 'pi05' else 'pi0', threads)
        ts = time_cpu_chunks(chunk, 2, warmup=1)
        cms = statistics.median(ts) * 1e3
        cpu = {'value': 1000.0 / cms, 'unit': 'chunks/s', 'cores': threads,
               'kind': chunk.kind,
               'sample': chunk.sample_doc() + '; median of 2 timed chunks '
                         'after 1 warm-up',
               'ms_per_chunk': cms}
        del chunk

    if rank == 0:
        line = {
            'metric': METRIC, 'value': world * 1000.0 / ms,
            'unit': 'chunks/s', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': ms,
            'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'bf16',
            'data': 'synthetic (seeded random bf16 weights of the real '
                    'architecture, seeded inputs)',
            'config': {'workload': workload_name(w), 'batch_per_gpu': 1,
                       'prefix_rows': E, 'suffix_rows': eng.S,
                       'euler_steps': len(eng.times),
                       'parallelism': f'replicas{world}',
                       'l2': 'no flush: every chunk streams ~6.6 GB of '
                             'weights (> 126 MB L2)'},
            'latency_ms': ms,
            'e2e': {'value': world * 1000.0 / e2e_ms, 'unit': 'chunks/s',
                    'latency_ms': e2e_ms, 'h2d_bytes_per_step': int(h2d),
                    'd2h_bytes_per_step': int(d2h)},
            'roofline': roof, 'roofline_prefill_gemm': roof_prefill,
            'cpu_baseline': cpu,
            'gpu_launches': int(eng.launches_per_call * args.steps),
            'launches_per_chunk': eng.launches_per_call,
            'clocks': clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_layer0(args, world, rank, local, dev, barrier, max_over_ranks):
    """config[0]: one Gemma-2B layer over 816 causal rows.  A step is one
    layer forward (one graph replay); value = layers/s (whole job)."""
    import torch.distributed as dist

    from fluxvla_b200.config import PI0Config
    from fluxvla_b200.layer import GemmaLayerB200
    from fluxvla_b200.weights import make_weights
    cfg = PI0Config(llm_layers=1)
    W = make_weights(cfg, seed=0, parts=('llm',), device=dev)
    del W['llm.embed']
    S = 816
    lay = GemmaLayerB200(cfg, W, S, device=dev)
    x = torch.randn(1, S, cfg.llm_width,
                    generator=torch.Generator().manual_seed(1 + rank)
                    ).pin_memory()
    lay.forward(x)
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        lay.replay()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.6)
    barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        lay.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = lay.forward(x)
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3 / args.steps)
    assert torch.isfinite(out).all()
    peaks, peak_kind = load_peaks()
    Wd, F, hd, H = cfg.llm_width, cfg.llm_mlp, cfg.head_dim, cfg.heads
    params = Wd * (H + 2) * hd + H * hd * Wd + 2 * Wd * F + F * Wd
    # causal attention: QK^T and PV over the visible half of the S x S map
    flops = 2.0 * S * params + 2 * 2 * H * hd * S * (S + 1) / 2
    tf = flops / (ms * 1e-3) / 1e12
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cms, kind, cores, sample = cpu_layer0_sample()
        cpu = {'value': 1000.0 / cms, 'unit': 'layers/s', 'cores': cores,
               'kind': kind, 'sample': sample, 'ms_per_layer': cms}
    if rank == 0:
        print(json.dumps({
            'metric': 'config[0] Gemma-2B layer forward (816 causal rows): '
                      'layers/s', 'value': world * 1000.0 / ms,
            'unit': 'layers/s', 'n_gpus': world, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': ms,
            'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
            'dtype': 'bf16', 'data': 'synthetic (seeded random bf16 weights, '
                                     'x ~N(0,1))',
            'config': {'workload': workload_name('layer0'), 'rows': S,
                       'parallelism': f'replicas{world}',
                       'l2': 'no flush: 220 MB of layer weights per step '
                             '(> 126 MB L2)'},
            'e2e': {'value': world * 1000.0 / e2e_ms, 'unit': 'layers/s',
                    'latency_ms': e2e_ms,
                    'h2d_bytes_per_step': S * Wd * 4,
                    'd2h_bytes_per_step': S * Wd * 4},
            'roofline': {'kernel': 'whole layer (7 launches)',
                         'bound': 'tensor', 'achieved': tf,
                         'peak': peaks['bf16_tflops'], 'unit': 'TFLOP/s',
                         'frac': tf / peaks['bf16_tflops'],
                         'peak_source': f'{peak_kind} burst bf16',
                         'algorithmic_flops': flops, 'traffic': None},
            'cpu_baseline': cpu,
            'gpu_launches': int(lay.launches_per_call * args.steps),
            'clocks': clocks}), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_serve(args, cfg, eng, n_tok, E, world, rank, local, dev):
    """config[4]: batches of independent config[2] requests (seeded per
    request) sharded round-robin over one replica per GPU; aggregate
    chunks/s and per-request p50/p99 latency (wall clock from the batch's
    release to the request's actions on the host, queueing included)."""
    import torch.distributed as dist

    from fluxvla_b200.serving import (ReplicaServer, dist_helpers,
                                      make_request, sweep)
    batches = [int(b) for b in args.batches.split(',') if b]
    server = ReplicaServer(eng)
    barrier, gather = dist_helpers(world, dev)
    cache = {}

    def request_of(i):
        if i not in cache:
            cache[i] = make_request(cfg, n_tok, i, seed_base=1000)
        return cache[i]
    # capture + warm-up on this rank's first request
    for _ in range(args.warmup):
        server.serve([request_of(rank)], 0.0)
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.6)
    res = sweep(server, request_of, batches, rank, world, barrier, gather)
    clocks = sampler.stop() if sampler else None
    if rank == 0:
        top = res[-1]
        print(json.dumps({
            'metric': 'PI0 serving sweep (config[4]): aggregate chunks/s and '
                      'p50/p99 request latency',
            'value': top['chunks_per_s'], 'unit': 'chunks/s', 'n_gpus': world,
            'steps': len(batches), 'warmup': args.warmup,
            'ms_per_step': 1000.0 * world / top['chunks_per_s'],
            'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': None,
            'dtype': 'bf16',
            'data': 'synthetic (seeded random bf16 weights; inputs seeded per '
                    'request = 1000 + index)',
            'config': {'workload': 'config[4]: PI0 serving sweep, config[2] '
                                   'requests, round-robin over one replica '
                                   'per GPU', 'batches': batches,
                       'prefix_rows': E, 'parallelism': f'replicas{world}'},
            'sweep': res, 'clocks': clocks,
            'gpu_launches': int(eng.launches_per_call *
                                sum(r['requests_per_gpu'] for r in res)),
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    ap.add_argument('--workload', default='pi0',
                    choices=['pi0', 'pi05', 'loop', 'serve', 'layer0'])
    ap.add_argument('--batches', default='1,4,16,64',
                    help='serve workload: batch sizes of the sweep')
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--depth', type=int, default=0,
                    help='profiling only: layers per tower (0 = full model)')
    ap.add_argument('--profile', action='store_true',
                    help='replay one chunk between cudaProfilerStart/Stop '
                         'and exit (for ncu --profile-from-start off)')
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == 'reference':
        return run_reference(args)
    return run_b200(args)


if __name__ == '__main__':
    sys.exit(main())
