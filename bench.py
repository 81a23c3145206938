"""Benchmark of the per-frame language-model path (talker + code predictor).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config q8_0|f32] [--impl reference]

Workload: Qwen3-TTS talker (28 layers) + code
predictor (5 layers, 15 heads), Q8_0 weights, batch 1, a 40-row N(0,1)
prompt, then K frames of streaming generation (K=156: the cache grows from
40 to ~196 positions).  Synthetic seeded weights of the real architecture
(no checkpoint here).  One step = one 80 ms frame = 1 talker step + 15
predictor steps + 16 heads with greedy choice.  --config f32 runs configs[0]
(f32 weights, 128 prior positions).

Arms
- default: libqtts.so on the GPU.  `value` = frames/s with everything
  resident in HBM: K frame kernels launched back to back
  (qtts_talker_run), CUDA events on the talker's stream.  `e2e` = the public
  API a caller uses (qtts_talker_start with the prompt from host memory, then
  qtts_talker_next_frame per frame, codes read back to the host each frame).
- --impl reference: the reference's CPU path, restated in C (oracle/; the
  reference's own Pascal code cannot be built here), timed on all host cores.

Multi-GPU (torchrun, one process per GPU): every GPU runs its own utterance
on a full weight replica, no data exchange (weak scaling); `value` = all
frames / the slowest rank's time.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mormot2-qwen-tts_b200")
sys.path.insert(0, PKG)

import synth  # noqa: E402

PROMPT_ROWS = {"q8_0": 40, "f32": 128}
SEED = 1
# bytes per frame of the weights read (talker + 15 predictor steps, heads and
# norms included), row-packed Q8_0 = 34 bytes per 32 weights
LAYER_CELLS = 1024 * (2 * 2048 + 2 * 1024 + 3 * 3072)
NORM_BYTES = (2 * 1024 + 2 * 128) * 4


def weight_bytes_per_frame(dtype, tl=28, pl=5, groups=16):
    per = (lambda cells: cells // 32 * 34) if dtype == "q8_0" else (lambda cells: cells * 4)
    talker = tl * (per(LAYER_CELLS) + NORM_BYTES) + 1024 * 4 + per(3072 * 1024)
    pred = pl * (per(LAYER_CELLS) + NORM_BYTES) + 1024 * 4 + per(2048 * 1024)
    return talker + (groups - 1) * pred


KV_POS_BYTES = 8 * 128 * 4 * 2  # K + V of one position in one layer (float32)


def kv_bytes_frame(talker_len, tl=28, pl=5, groups=16):
    """KV bytes read + written by one frame whose talker step is at position
    talker_len (cache already holding talker_len positions)."""
    t = tl * KV_POS_BYTES * (talker_len + 1)
    p = 0
    for g in range(groups - 1):
        rows = 2 if g == 0 else 1
        prior = 0 if g == 0 else g + 1
        p += pl * KV_POS_BYTES * (prior + rows)
    return t + p


def oracle_module():
    """oracle/oracle.py (the CPU restatement's wrapper), imported by path:
    only the cpu_baseline and reference legs use it, as the checker."""
    import importlib.util
    if "qtts_oracle_wrapper" not in sys.modules:
        spec = importlib.util.spec_from_file_location("qtts_oracle_wrapper", os.path.join(ROOT, "oracle", "oracle.py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules["qtts_oracle_wrapper"] = mod
        spec.loader.exec_module(mod)
    return sys.modules["qtts_oracle_wrapper"]


def measured_peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        return None


# the sources of the batch-1 frame kernel (qtts::decode_kernel and the
# sampler it inlines): a profile of that kernel names the build by them
DECODE_SOURCES = ("qtts_decode.cuh", "qtts_sample.cuh")


def source_digest(files=DECODE_SOURCES):
    """sha256 (first 16 hex digits) of the named kernel sources under csrc/:
    names the build of a kernel a profile was captured on."""
    import hashlib
    h = hashlib.sha256()
    for name in sorted(files):
        h.update(name.encode())
        h.update(open(os.path.join(PKG, "csrc", name), "rb").read())
    return h.hexdigest()[:16]


def ncu_traffic(config):
    """DRAM bytes per launch of the frame kernel from an ncu capture of THIS
    build (profiles/decode_kernel_<config>_frame.md records the source
    digest it was captured on and the measured bytes), else None: a figure
    measured on other code is not reported."""
    path = os.path.join(ROOT, "profiles", f"decode_kernel_{config}_frame.md")
    got = {}
    try:
        for line in open(path):
            for key in ("traffic_bytes_per_launch:", "source_digest:"):
                if line.startswith(key):
                    got[key] = line.split(":", 1)[1].strip()
    except OSError:
        return None
    if got.get("source_digest:") != source_digest() or "traffic_bytes_per_launch:" not in got:
        return None
    return float(got["traffic_bytes_per_launch:"])


class Clocks:
    """SM clocks and clock-event reasons sampled DURING the timed region: an
    NVML thread (read-only queries) every 2 ms, so that a region of tens of
    milliseconds still holds samples; nvidia-smi -lms 200 where NVML cannot
    be loaded.  start() returns once the first sample is in."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index):
        import threading
        self.index, self.p, self.nvml, self.samples = index, None, None, []
        self.done = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = self._handle(pynvml, index)
            self.mx = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.bits = [pynvml.nvmlClocksEventReasonHwSlowdown, pynvml.nvmlClocksEventReasonHwThermalSlowdown,
                         pynvml.nvmlClocksEventReasonSwThermalSlowdown, pynvml.nvmlClocksEventReasonSwPowerCap]
            self._sample()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception:
            self.nvml = None
            try:
                self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={self.Q}",
                                           "--format=csv,noheader,nounits", "-lms", "200"],
                                          stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except OSError:
                self.p = None

    @staticmethod
    def _handle(pynvml, index):
        # the CUDA device's own board (CUDA and NVML may number GPUs apart)
        try:
            import torch
            pr = torch.cuda.get_device_properties(index)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(index)

    def _sample(self):
        pn = self.nvml
        sm = pn.nvmlDeviceGetClockInfo(self.h, pn.NVML_CLOCK_SM)
        r = pn.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        self.samples.append((float(sm), float(self.mx), {n for n, b in zip(self.NAMES, self.bits) if r & b}))

    def _run(self):
        while not self.done.wait(0.002):
            try:
                self._sample()
            except Exception:
                return

    def stop(self):
        if self.nvml:
            self.done.set()
            self.t.join(timeout=5)
            try:
                self._sample()  # the end of the region
            except Exception:
                pass
            rows = self.samples
        elif self.p:
            self.p.terminate()
            try:
                out, _ = self.p.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
                out, _ = self.p.communicate()
            rows = []
            for line in out.splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) < 8:
                    continue
                try:
                    rows.append((float(f[1]), float(f[2]),
                                 {n for n, v in zip(self.NAMES, f[4:8]) if v.lower().startswith("active")}))
                except ValueError:
                    continue
        else:
            return None
        if not rows:
            return None
        reasons = set().union(*(r[2] for r in rows))
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows),
                "source": "NVML, every 2 ms during the timed region" if self.nvml else "nvidia-smi -lms 200"}


def build_host_model(dtype, seed=SEED, tlayers=28, players=5):
    t0 = time.time()
    tl, tf = synth.stack(seed, "talker", tlayers)
    pl, pf = synth.stack(seed, "predictor", players)
    m = dict(tl=tl, tf=tf, pl=pl, pf=pf, th=synth.talker_head(seed), ph=synth.predictor_heads(seed),
             ce=synth.codec_embedding(seed), pe=synth.predictor_embeddings(seed),
             pad=synth.text_rows(seed, 1, key=1)[0])
    m["gen_s"] = time.time() - t0
    return m


def cpu_frames(m, dtype, prompt, frames, threads=None, seconds=None, warmup=0):
    """The oracle on host cores: prefill and `warmup` frames (untimed), then
    up to `frames` frames, stopping early once `seconds` have passed (after 2
    frames); returns (seconds, frames done, threads used)."""
    O = oracle_module()
    if threads:
        O.set_threads(threads)
    ts = O.OraStack(synth.CONFIG, m["tl"], m["tf"], dtype)
    ps = O.OraStack(synth.CONFIG, m["pl"], m["pf"], dtype)
    th = O.OraHeads(synth.HIDDEN, dtype)
    th.add(m["th"])
    ph = O.OraHeads(synth.HIDDEN, dtype)
    for h in m["ph"]:
        ph.add(h)
    tlm = O.OraLm(ts, th, prompt.shape[0] + frames + warmup + 8)
    plm = O.OraLm(ps, ph, 32)
    tk = O.OraTalker(tlm, th, plm, ph, m["ce"], m["pe"], synth.CODEC_EOS)
    tk.start(prompt, None, m["pad"])
    codes = np.zeros(16, np.int32)
    for _ in range(warmup):
        if not tk.next_frame(codes):
            tk.start(prompt, None, m["pad"])
    tk.start(prompt, None, m["pad"])
    done = 0
    t0 = time.perf_counter()
    for _ in range(frames):
        if not tk.next_frame(codes):
            tk.start(prompt, None, m["pad"])
            continue
        done += 1
        if seconds is not None and done >= 2 and time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    n = O.threads()
    for o in (tk, tlm, plm, ts, ps, th, ph):
        o.free()
    return dt, done, n


def cpu_sample(dtype, seconds=15.0, threads=None):
    """The bounded CPU sample of cpu_baseline: the oracle (the C restatement
    of the reference CPU path) on `threads` host threads (default: all),
    about `seconds` of frames after the utterance's prefill.  Runs in a
    process of its own (bench.py --cpu-sample), so that no GPU context, no
    process group and no OMP_NUM_THREADS inherited from a launcher shares the
    cores with it."""
    env = dict(os.environ)
    n = threads or os.cpu_count()
    env["OMP_NUM_THREADS"] = str(n)
    env.pop("OMP_PROC_BIND", None)
    env.pop("OMP_PLACES", None)
    r = subprocess.run([sys.executable, os.path.abspath(__file__), "--cpu-sample", dtype, "--cpu-seconds",
                        str(seconds)], env=env, capture_output=True, text=True, timeout=600)
    if r.returncode != 0:
        return {"error": (r.stderr or r.stdout).strip()[-300:]}
    return json.loads(r.stdout.strip().splitlines()[-1])


def cpu_sample_main(dtype, seconds):
    m = build_host_model(dtype)
    prompt = synth.config1_prompt(SEED, PROMPT_ROWS[dtype])
    dt, done, used = cpu_frames(m, dtype, prompt, 156, seconds=seconds)
    print(json.dumps({"value": done / dt, "unit": "frames/s", "cores": used, "kind": "port",
                      "sample": f"{done} frames of the configs[1] utterance after its prefill, {dt:.1f} s (C "
                                "restatement of the reference CPU path, AVX2+FMA, OpenMP over output rows, "
                                f"{used} threads, own process)"}), flush=True)


def max_over_ranks(values, dist, device):
    """Each of `values` (timings of this rank) replaced by its maximum over
    the ranks of the job (the values themselves without a process group):
    the job's time is that of its slowest rank."""
    import torch
    if not dist:
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]


def job_value(world, units, ms):
    """Whole-job throughput: the units every rank processed over the
    max-over-ranks time (weak scaling: each rank does `units`)."""
    return world * units / (ms / 1000.0)


def reference_arm(args, rank):
    if rank != 0:
        return
    dtype = args.config
    m = build_host_model(dtype)
    prompt = synth.config1_prompt(SEED, PROMPT_ROWS[dtype])
    cores = os.cpu_count()
    # W warm-up frames, then K timed frames (each step = one frame on the CPU)
    dt, done, used = cpu_frames(m, dtype, prompt, args.steps, cores, warmup=args.warmup)
    fps = done / dt
    line = {
        "impl": "reference",
        "metric": metric_name(dtype), "value": fps, "unit": "frames/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dt / max(done, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype_name(dtype),
        "data": "synthetic (seeded N(0,0.02) weights of the Qwen3-TTS talker/predictor architecture)",
        "config": config_dict(dtype, args),
        "cpu_baseline": {"value": fps, "unit": "frames/s", "cores": used, "kind": "port",
                         "sample": f"{done} frames of the {PROMPT_ROWS[dtype]}-row-prompt utterance after its prefill "
                                   "(C restatement of the reference CPU path, AVX2+FMA, OpenMP)"},
        "e2e": {"value": fps, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def metric_name(dtype):
    return f"talker+predictor frames/s @B=1 per GPU ({'Q8_0' if dtype == 'q8_0' else 'f32'}; ms/frame = ms_per_step)"


def dtype_name(dtype):
    return "q8_0 weights x f32 activations (f32 accumulate)" if dtype == "q8_0" else "f32"


def config_dict(dtype, args):
    extra = {} if (args.talker_layers, args.pred_layers) == (28, 5) else {
        "layers_override": f"talker {args.talker_layers}, predictor {args.pred_layers} (profiling case, not a bench line)"}
    return {**extra, "workload": ("configs[1]: Q8_0, batch 1 per GPU, 40-row N(0,1) prompt, then K streaming frames"
                         if dtype == "q8_0" else "configs[0]: f32, batch 1 per GPU, 128 prior positions, then K frames"),
            "model": "Qwen3-TTS-12Hz-0.6B talker (28 layers) + code predictor (5 layers, 15 heads), synthetic weights",
            "global_batch": args.gpus, "frames": args.steps, "prompt_rows": PROMPT_ROWS[dtype],
            "parallelism": f"replicas x{args.gpus} (independent utterances, no collective)",
            "l2": "working set per frame (weights) larger than L2: no flush needed"}


BATCH_CTX = (50, 1000)  # configs[2]: per-utterance context drawn uniformly
KV_POS_BF16 = 8 * 128 * 2 * 2  # K + V of one position in one layer (bf16)


BOX_BATCH = 128       # configs[4]: concurrent utterances per GPU
BOX_PROMPT = (20, 80)  # configs[4]: prompt rows
BOX_FRAMES = 300       # configs[4]: frames per utterance


def batched_frames(args, qtts, torch, tstack, th, pstack, ph, m, local_rank, rank, dist):
    """B utterances (default 64) decoded together,
    Q8_0 weights, contexts drawn uniformly in [50, 1000] (prefilled through
    the batched path), paged bf16 KV cache; one step = one frame of every
    utterance (15 batched predictor steps + 1 batched talker step) through
    qtts_talkers_next_frame, codes read back to the host each frame.

    """
    B, K, W = args.batch, args.batch_steps, 3
    lo, hi = args.batch_ctx
    ctx = synth.config2_contexts(SEED, B, lo, hi, rank)
    chunk = 16384
    tb = qtts.QwenBatch(tstack, th, max_seqs=B, max_tokens=chunk, max_pos=hi + K + W + 8, kv_dtype="bf16")
    pb = qtts.QwenBatch(pstack, ph, max_seqs=B, max_tokens=2 * B, max_pos=16, kv_dtype="bf16")
    ts = qtts.QwenTalkers(tb, pb, m["ce"], m["pe"], synth.CODEC_EOS)
    stream = torch.cuda.ExternalStream(ts.stream, device=torch.device("cuda", local_rank))
    t0 = time.perf_counter()
    i = 0
    while i < B:
        j, rows = i, 0
        while j < B and rows + ctx[j] <= chunk:
            rows += int(ctx[j])
            j += 1
        ts.start(list(range(i, j)), [synth.config2_prompt(s, int(ctx[s]), SEED) for s in range(i, j)],
                 [None] * (j - i), m["pad"])
        i = j
    prefill_s = time.perf_counter() - t0
    seqs = list(range(B))
    for _ in range(W):
        ts.next_frame(seqs)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    frames = 0
    for _ in range(K):
        _, more = ts.next_frame(seqs)
        frames += int(more.sum())
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks([e0.elapsed_time(e1)], dist, "cpu")[0]
    world = dist.get_world_size() if dist else 1
    ts.free()
    tb.free()
    pb.free()
    # algorithmic bytes of one batched frame: the weights once, the talker KV
    # of every utterance (bf16), the predictor KV
    tl, pl = args.talker_layers, args.pred_layers
    wb = weight_bytes_per_frame("q8_0", tl, pl)
    mean_ctx = float(ctx.mean()) + W + K / 2.0
    kv = tl * KV_POS_BF16 * B * (mean_ctx + 1)
    kv += sum(pl * KV_POS_BF16 * B * ((0 if g == 0 else g + 1) + (2 if g == 0 else 1)) for g in range(15))
    peaks = measured_peaks()
    peak = peaks["hbm_gbs"] if peaks else 6650.0
    achieved = (wb + kv) / (ms / 1000.0 / K) / 1e9
    extra = {} if (tl, pl) == (28, 5) else {"layers_override": f"talker {tl}, predictor {pl} (profiling case)"}
    workload = (f"configs[2]: {B} utterances per GPU, contexts U({lo},{hi}), Q8_0 weights, "
                "paged bf16 KV (16-position pages), fp16 activations on the tcgen05 GEMMs")
    return {**extra,
            "workload": workload,
            "metric": "frames/s per GPU @B=%d" % B if world == 1 else "frames/s of all GPUs @B=%d per GPU" % B,
            "value": job_value(world, frames, ms), "unit": "frames/s", "steps": K, "warmup": W,
            "ms_per_batched_frame": ms / K, "frames": frames, "prefill_s_rank0": prefill_s,
            "mean_ctx": float(ctx.mean()),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "algorithmic_bytes_per_batched_frame": wb + kv, "traffic": None,
                         "what": "whole batched frame (weights once + talker/predictor KV), CUDA events on the stream"},
            "e2e_note": "timed through qtts_talkers_next_frame (the public call), codes of every frame read back to "
                        "the host inside the timed region; the prefill is outside it"}


def sum_over_ranks(values, dist):
    """Each of `values` summed over the ranks of the job (gloo, CPU)."""
    import torch
    if not dist:
        return [float(v) for v in values]
    t = torch.tensor([float(v) for v in values], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return [float(v) for v in t]


def box_run(args, qtts, torch, tstack, th, pstack, ph, m, local_rank, rank, dist):
    """BASELINE.json configs[4], the whole run: 1024 independent utterances
    of up to 300 frames, prompts of U(20, 80) N(0,1) rows, Q8_0 weights,
    paged bf16 KV, at most 128 concurrent utterances per GPU.  Rank r of N
    takes utterances r, r + N, ...; its 128 slots start with its first 128,
    and a slot whose utterance ends (codec EOS, or its 300th frame) takes the
    next one (TQwenTalker.Start on the freed slot; a frame's admissions in
    one call).  Timed: from the first admission to the last frame, CUDA
    events on the talkers' stream, max over ranks; value = the frames of
    every utterance of the box over that time.  The prompt rows are made on
    the host before the timed region; their upload (inside Start) and every
    frame's codes (read back) are in it."""
    import collections
    world = dist.get_world_size() if dist else 1
    U, F = args.box_utterances, args.box_frames
    mine = list(range(rank, U, world))
    B = min(BOX_BATCH, len(mine))
    lens = synth.config4_lengths(SEED, U, BOX_PROMPT[0], BOX_PROMPT[1])
    prompts = {u: synth.config4_prompt(u, int(lens[u]), SEED) for u in mine}
    tb = qtts.QwenBatch(tstack, th, max_seqs=B, max_tokens=B * BOX_PROMPT[1], max_pos=BOX_PROMPT[1] + F + 16,
                        kv_dtype="bf16")
    pb = qtts.QwenBatch(pstack, ph, max_seqs=B, max_tokens=2 * B, max_pos=16, kv_dtype="bf16")
    ts = qtts.QwenTalkers(tb, pb, m["ce"], m["pe"], synth.CODEC_EOS)
    stream = torch.cuda.ExternalStream(ts.stream, device=torch.device("cuda", local_rank))
    # warm-up: 3 frames of the first utterances (the timed run starts them again)
    ts.start(list(range(B)), [prompts[u] for u in mine[:B]], [None] * B, m["pad"])
    for _ in range(3):
        ts.next_frame(list(range(B)))
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    tl, pl = args.talker_layers, args.pred_layers
    pred_kv = sum(pl * KV_POS_BF16 * ((0 if g == 0 else g + 1) + (2 if g == 0 else 1)) for g in range(15))
    queue = collections.deque(mine)
    slot_utt, slot_frames, slot_ctx = [-1] * B, [0] * B, [0] * B
    calls = {"start": 0, "next_frame": 0}

    def admit(slots):
        take = []
        for s in slots:
            if not queue:
                break
            u = queue.popleft()
            slot_utt[s], slot_frames[s], slot_ctx[s] = u, 0, int(lens[u])
            take.append(s)
        if take:
            ts.start(take, [prompts[slot_utt[s]] for s in take], [None] * len(take), m["pad"])
            calls["start"] += 1

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    admit(range(B))
    frames, eos, kv_bytes = 0, 0, 0.0
    while True:
        active = [s for s in range(B) if slot_utt[s] >= 0]
        if not active:
            break
        _, more = ts.next_frame(active)
        calls["next_frame"] += 1
        freed = []
        for s, mo in zip(active, more):
            kv_bytes += tl * KV_POS_BF16 * (slot_ctx[s] + 1) + pred_kv
            slot_ctx[s] += 1
            if mo:
                slot_frames[s] += 1
                frames += 1
            else:
                eos += 1
            if not mo or slot_frames[s] >= F:
                slot_utt[s] = -1
                freed.append(s)
        if freed:
            admit(freed)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks([e0.elapsed_time(e1)], dist, "cpu")[0]
    tot_frames, tot_eos, tot_batched, tot_kv = sum_over_ranks([frames, eos, calls["next_frame"], kv_bytes], dist)
    ts.free()
    tb.free()
    pb.free()
    wb = weight_bytes_per_frame("q8_0", tl, pl)
    # algorithmic bytes of the whole box: the weights once per batched frame
    # of every rank, the KV of every utterance frame
    algo = wb * tot_batched + tot_kv
    peaks = measured_peaks()
    peak = peaks["hbm_gbs"] if peaks else 6650.0
    achieved = algo / (ms / 1000.0) / 1e9 / world  # per GPU, against one GPU's peak
    return {"workload": f"configs[4]: {U} utterances of up to {F} frames, prompts U{BOX_PROMPT} N(0,1) rows, "
                        f"at most {BOX_BATCH} concurrent per GPU (slots refilled as utterances end), Q8_0 "
                        "weights, paged bf16 KV, fp16 activations on the tcgen05 GEMMs; the whole run",
            "metric": "box frames/s (all GPUs)", "value": tot_frames / (ms / 1000.0), "unit": "frames/s",
            "ms_total": ms, "frames": int(tot_frames), "eos_endings": int(tot_eos),
            "batched_frames_rank0": calls["next_frame"], "start_calls_rank0": calls["start"],
            "utterances": U, "utterances_rank0": len(mine),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "algorithmic_bytes": algo, "traffic": None,
                         "what": "the whole run per GPU (weights once per batched frame + KV of every utterance "
                                 "frame), CUDA events on the stream, max over ranks"},
            "timing": "CUDA events on the talkers' stream around the whole run (admissions with their prompt "
                      "uploads, every batched frame with its codes read back), max over ranks"}


PREFILL_LEN = (256, 2048)  # configs[3]: prompt lengths drawn uniformly
PREFILL_SEQS = 16


def prefill_measure(args, qtts, torch, m, dev, rank):
    """one batched prefill of 16 prompts of
    U(256, 2048) N(0,1) rows through the 28-layer talker with float32
    weights (tcgen05 projections with fp16 activations, causal attention in
    f32) and its head on the last rows; each step resets the sequences and
    runs qtts_batch_forward from host memory (the rows up, the logits and
    normed states back)."""
    lens = synth.config3_lengths(SEED, PREFILL_SEQS, PREFILL_LEN[0], PREFILL_LEN[1], rank)
    T = int(lens.sum())
    th = qtts.QwenLmHeads(dev, "talker", synth.HIDDEN, "f32")
    th.add(m["th"])
    st = qtts.qwen_lm_stack(dev, synth.CONFIG, m["tl"], m["tf"], "f32")
    b = qtts.QwenBatch(st, th, max_seqs=PREFILL_SEQS, max_tokens=T, max_pos=PREFILL_LEN[1], kv_dtype="f32")
    x = np.concatenate([synth.config3_prompt(i, int(n), SEED) for i, n in enumerate(lens)])
    x = torch.from_numpy(x).pin_memory().numpy()
    seqs = np.arange(PREFILL_SEQS)

    def step():
        for q in range(PREFILL_SEQS):
            b.reset(q)
        b.forward(seqs, lens, x)

    step()  # warm-up
    torch.cuda.synchronize()
    K = max(1, args.prefill_steps)
    t0 = time.perf_counter()
    for _ in range(K):
        step()
    dt = (time.perf_counter() - t0) / K
    b.free()
    qtts.stack_destroy(st)
    th.free()
    # FLOPs of one prefill: the projections of every row (2 per weight) and
    # causal attention (QK and PV, 2 x 2 per query head, key and dim)
    L = len(m["tl"])
    proj = 2.0 * LAYER_CELLS * L * T + 2.0 * 3072 * 1024 * PREFILL_SEQS
    att = L * 16 * 128 * 4.0 * float(sum(int(n) * (int(n) + 1) // 2 for n in lens))
    peaks = measured_peaks()
    peak = peaks["bf16_tflops"] if peaks else 1590.0
    achieved = (proj + att) / dt / 1e12
    return {"workload": f"configs[3]: prefill of {PREFILL_SEQS} prompts U({PREFILL_LEN[0]},{PREFILL_LEN[1]}) rows "
                        f"({T} rows), {L}-layer talker, f32 weights, fp16 activations, f32 softmax, f32 KV",
            "metric": "prefill tokens/s per GPU", "value": T / dt, "unit": "tokens/s", "ms_per_step": dt * 1000.0,
            "steps": K, "rows": T,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "flops_per_step": proj + att, "attention_flops": att,
                         "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops)" if peaks else "fallback"},
            "timing": "host wall clock around qtts_batch_forward (rows from pinned host memory, logits back)"}


# the phases of the frame kernel as its trace marks them (qtts_decode.cuh
# Compute::mark): (from tag, to tag) -> phase; 100 + b / 200 + b = arrival at /
# departure from barrier b
TRACE_PHASES = {
    (10, 11): "QKV GEMV (P1)", (11, 21): "attention, polling its rows (P2)",
    (202, 30): "combine of the splits (P3)", (30, 31): "O GEMV + residual (P3)", (21, 31): "O GEMV by kv head",
    (203, 40): "RMSNorm staging (P4)", (40, 41): "gate/up GEMV + SwiGLU (P4)", (204, 50): "staging (P5)",
    (50, 51): "down GEMV + residual (P5)", (205, 10): "RMSNorm staging (P1)", (60, 61): "head GEMV + argmax keys",
    (206, 10): "argmax + next input (P1 staging)", (51, 10): "RMSNorm staging, polling the residual (P1)",
    (61, 10): "argmax keys polled + next input (P1 staging)",
}
# Q8_0 bytes a GEMV phase streams (row-packed, 34 B per 32 weights)
TRACE_BYTES = {"QKV GEMV (P1)": 4096 * 1088, "O GEMV + residual (P3)": 1024 * 2176, "O GEMV by kv head": 8192 * 272,
               "gate/up GEMV + SwiGLU (P4)": 6144 * 1088, "down GEMV + residual (P5)": 1024 * 3264}


def trace_measure(qtts, tk):
    """The phase trace of one configs[1] frame (qtts_talker_trace_frame:
    CTA 0's timestamps at each phase boundary), the fastest of 5 traced
    frames after 20 untraced ones: mean time of each phase over the
    predictor's 75 layer steps and the talker's 28 layers, barriers apart,
    and each GEMV phase's weight bytes over its time (GB/s; the talker's
    weights stream from HBM, the predictor's are L2 hits)."""
    codes = np.zeros(16, np.int32)
    for _ in range(20):
        tk.next_frame(codes)
    best = None
    for _ in range(5):
        _, st = tk.trace_frame(codes)
        if best is None or st[-1][1] - st[0][1] < best[-1][1] - best[0][1]:
            best = st
    st = best
    heads = [i for i, (t, _) in enumerate(st) if t == 61]
    split = heads[14]  # the 15th predictor head ends the predictor part
    out = {"frame_us": (st[-1][1] - st[0][1]) / 1000.0}
    peaks = measured_peaks()
    peak = peaks["hbm_gbs"] if peaks else 6650.0
    for name, lo, hi in (("predictor", 0, split + 1), ("talker", split, len(st))):
        agg, bars = {}, {}
        for i in range(lo + 1, hi):
            a, b = st[i - 1][0], st[i][0]
            d = st[i][1] - st[i - 1][1]
            if 100 < a < 200 and b == a + 100:
                bars.setdefault(f"barrier {a - 100}", []).append(d)
            elif (a, b) in TRACE_PHASES:
                agg.setdefault(TRACE_PHASES[(a, b)], []).append(d)
        part = {"us": (st[hi - 1][1] - st[lo][1]) / 1000.0, "phases_us": {}, "barriers_us": {}, "gemv_gbs": {}}
        for k, v in agg.items():
            part["phases_us"][k] = round(float(np.mean(v)) / 1000.0, 3)
            if k in TRACE_BYTES:
                gbs = TRACE_BYTES[k] / float(np.mean(v))
                part["gemv_gbs"][k] = {"gb_s": round(gbs, 1), "frac_of_hbm": round(gbs / peak, 4)}
        for k, v in bars.items():
            part["barriers_us"][k] = {"mean": round(float(np.mean(v)) / 1000.0, 3), "count": len(v)}
        out[name] = part
    return out


def start_prompt_measure(qtts, tk, dev, cpu_leg):
    """TQwenTalker.Start (talker.pas:471-592) from token ids on the device
    (qtts_talker_start_prompt: 32 text tokens, streaming, a voice; the text
    projection of every prompt row, the codec rows, the talker's prefill and
    the first ChooseCode0), host wall clock around the synchronous call.
    With cpu_leg, the same rows restated on the host cores (the reference
    builds them with TextProject on the CPU) are timed beside it.  A
    synthetic 4096-row BF16 text table stands for the 151,936-row one: Start
    only gathers its prompt's rows."""
    rng = np.random.default_rng(SEED + 7)
    th, hid, vocab = 2048, synth.HIDDEN, 4096
    emb = (rng.standard_normal((vocab, th)) * 0.05).astype(np.float32)
    bits = (emb.view(np.uint32) >> 16).astype(np.uint16)
    emb = (bits.astype(np.uint32) << 16).view(np.float32)
    w1 = (rng.standard_normal((th, th)) * 0.02).astype(np.float32)
    b1 = (rng.standard_normal(th) * 0.02).astype(np.float32)
    w2 = (rng.standard_normal((hid, th)) * 0.02).astype(np.float32)
    b2 = (rng.standard_normal(hid) * 0.02).astype(np.float32)
    tp = qtts.QwenTextProject(dev, bits, w1, b1, w2, b2)
    tok = qtts.PromptTokens(4093, 4094, 4095, 2148, 2149)
    ids = [4000, 4001, 4002] + [int(v) for v in rng.integers(0, 3990, 32)] + [4003, 4002, 4000, 4001, 4002]
    codec = [2155, 2156, 2157, 3065, 2148, 2149]
    try:
        for _ in range(3):
            tk.start_prompt(tp, tok, ids, codec)
        n = 20
        t0 = time.perf_counter()
        for _ in range(n):
            tk.start_prompt(tp, tok, ids, codec)
        ms = (time.perf_counter() - t0) * 1000.0 / n
        rows, trailing = tk.prompt_rows(tp, tok, ids, codec)
        out = {"ms_per_start": ms, "prefill_rows": int(rows.shape[0]), "trailing_rows": int(trailing.shape[0]),
               "text_tokens": 32,
               "includes": "qtts_talker_start_prompt: ids up, text projection (fc1 2048x2048 + SiLU + fc2) of "
                           "every row with the codec rows added, 28-layer prefill, first ChooseCode0",
               "timing": "host wall clock around the synchronous call, 20 calls after 3"}
        if cpu_leg:
            O = oracle_module()
            toks = {"tts_bos": 4093, "tts_eos": 4094, "tts_pad": 4095, "codec_pad": 2148, "codec_bos": 2149}
            ce = synth.codec_embedding(SEED)
            t0 = time.perf_counter()
            O.start_rows(emb, w1, b1, w2, b2, ce, toks, ids, codec)
            out["cpu_baseline_rows_ms"] = (time.perf_counter() - t0) * 1000.0
            out["cpu_baseline_kind"] = "port: the rows alone (no prefill), C restatement, one thread"
        return out
    finally:
        tp.free()


def heads_load_measure(qtts, dev, m, cpu_leg):
    """TQwenLmHeads.Add of the 15 predictor heads from a BF16 safetensors
    file, converted to Q8_0 (the conversion ParallelQ8MatchesSerial times,
    tests/test.tts.qwen.talker.pas:256-304): qtts_heads_add_safetensors reads
    the rows in place and quantises them on the device.  Host wall clock,
    the file in the page cache (one untimed pass first)."""
    import shutil
    import tempfile

    import torch
    from safetensors.torch import save_file
    d = tempfile.mkdtemp(prefix="qtts_heads_")
    try:
        path = os.path.join(d, "heads.safetensors")
        names = [f"talker.code_predictor.lm_head.{g}.weight" for g in range(len(m["ph"]))]
        save_file({n: torch.from_numpy(h).to(torch.bfloat16) for n, h in zip(names, m["ph"])}, path)
        runs = []
        for _ in range(4):
            f = qtts.SafeTensorsFile(path)
            t0 = time.perf_counter()
            h = qtts.QwenLmHeads(dev, "predictor", synth.HIDDEN, "q8_0")
            for n in names:
                h.add_file(f, n, synth.PRED_VOCAB)
            runs.append((time.perf_counter() - t0) * 1000.0)
            crc = h.digest()  # after the timer, as the reference's test reads it
            h.free()
            f.close()
        out = {"ms": min(runs[1:]), "heads": len(names), "rows": synth.PRED_VOCAB, "hidden": synth.HIDDEN,
               "bf16_bytes": os.path.getsize(path), "crc32c": "%08x" % crc,
               "timing": "host wall clock around heads create + 15 x qtts_heads_add_safetensors (each "
                         "synchronous), the file opened before and the digest read after, as the reference's "
                         "test times it; best of 3 after 1"}
        if cpu_leg:
            O = oracle_module()
            t0 = time.perf_counter()
            for hm in m["ph"]:
                O.quantize_q8_0(torch.from_numpy(hm).to(torch.bfloat16).float().numpy())
            out["cpu_baseline_ms"] = (time.perf_counter() - t0) * 1000.0
            out["cpu_baseline_kind"] = "port: ggml quantize_row_q8_0_ref restated in C, one thread, rows widened first"
        return out
    finally:
        shutil.rmtree(d, ignore_errors=True)


def codec_measure(qtts, dev, cpu_leg):
    """The 12 Hz decoder (TQwenCodec.Decode, codec.pas:1019-1038) on the
    device, seeded weights read from a safetensors file: 50 frames decoded
    one call per frame (the streaming use, each call synchronous) and the
    same 50 frames in one call; host wall clock.  One frame is 80 ms of
    audio, so real time is 12.5 frames/s.  With cpu_leg, the C restatement
    decodes 4 frames in one call on the host cores beside it."""
    import shutil
    import tempfile

    from safetensors.numpy import save_file
    w = synth.codec_weights(SEED)
    d = tempfile.mkdtemp(prefix="qtts_codec_")
    try:
        path = os.path.join(d, "codec.safetensors")
        save_file(w, path)
        f = qtts.SafeTensorsFile(path)
        c = qtts.QwenCodec(dev, f)
        try:
            codes = np.random.default_rng(SEED + 11).integers(0, 2048, (50, 16)).astype(np.int32)
            c.decode(codes[:8])  # work buffers grown, kernels loaded
            c.reset()
            t0 = time.perf_counter()
            for i in range(50):
                c.decode(codes[i:i + 1])
            ms_stream = (time.perf_counter() - t0) * 1000.0 / 50
            c.reset()
            c.decode(codes)  # the work buffers of a 50-frame call
            c.reset()
            t0 = time.perf_counter()
            c.decode(codes)
            ms_call = (time.perf_counter() - t0) * 1000.0 / 50
        finally:
            c.free()
            f.close()
        out = {"ms_per_frame_streaming": ms_stream, "ms_per_frame_50_per_call": ms_call,
               "frames_per_s_streaming": 1000.0 / ms_stream, "realtime_factor_streaming": 80.0 / ms_stream,
               "timing": "host wall clock around qtts_codec_decode (codes up, samples back), 50 frames after 8",
               "kernels": "tcgen05 products with float32 accuracy (3xTF32: tf32 hi/lo split of both operands, "
                          "3 MMAs) over im2col rows for every convolution and projection, K cut into fixed chunks "
                          "of 256 on their own CTAs, partials summed in chunk order"}
        if cpu_leg:
            O = oracle_module()
            oc = O.OraCodec(w)
            t0 = time.perf_counter()
            oc.decode(codes[:4])
            out["cpu_baseline_ms_per_frame"] = (time.perf_counter() - t0) * 1000.0 / 4
            out["cpu_baseline_kind"] = "port: C restatement of TQwenCodec, AVX2, OpenMP, 4 frames in one call"
            oc.free()
        return out
    finally:
        shutil.rmtree(d, ignore_errors=True)


def summary(line):
    """The headline figures of every measurement in the line, compact (the
    configs[2]-[4] numbers sit in long nested objects)."""
    def pick(d, *keys):
        for k in keys:
            if not isinstance(d, dict) or k not in d:
                return None
            d = d[k]
        return round(d, 4) if isinstance(d, float) else d
    return {"b1_frames_s": pick(line, "value"), "b1_ms_per_frame": pick(line, "ms_per_step"),
            "b1_hbm_frac": pick(line, "roofline", "frac"), "b1_e2e_frames_s": pick(line, "e2e", "value"),
            "cpu_frames_s": pick(line, "cpu_baseline", "value"),
            "b64_frames_s": pick(line, "batched", "value"), "b64_hbm_frac": pick(line, "batched", "roofline", "frac"),
            "box_frames_s": pick(line, "box", "value"), "box_hbm_frac": pick(line, "box", "roofline", "frac"),
            "prefill_tokens_s": pick(line, "prefill", "value"),
            "prefill_tensor_frac": pick(line, "prefill", "roofline", "frac"),
            "codec_ms_per_frame_streaming": pick(line, "codec", "ms_per_frame_streaming")}


def gpu_arm(args, rank, world, local_rank):
    import torch
    import qtts
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        # the harness only: a barrier around the timed regions and the max of
        # the ranks' timings.  Nothing of the path crosses devices (each rank
        # decodes its own utterances), so gloo on the host serves it.
        import datetime
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=900))
    if args.only_codec:
        # the codec leg alone (profiling runs): no language-model weights
        dev = qtts.QwenDevice(local_rank)
        if rank == 0:
            print(json.dumps({"impl": "ours", "codec": codec_measure(qtts, dev, False)}), flush=True)
        dev.close()
        if dist:
            dist.destroy_process_group()
        return
    dtype = args.config
    m = build_host_model(dtype, tlayers=args.talker_layers, players=args.pred_layers)
    prompt = synth.config1_prompt(SEED, PROMPT_ROWS[dtype], rank)
    K, W = args.steps, args.warmup
    dev = qtts.QwenDevice(local_rank)
    th = qtts.QwenLmHeads(dev, "talker", synth.HIDDEN, dtype)
    th.add(m["th"])
    ph = qtts.QwenLmHeads(dev, "predictor", synth.HIDDEN, dtype)
    for h in m["ph"]:
        ph.add(h)
    max_pos = PROMPT_ROWS[dtype] + max(K, W) + 16
    tstack = qtts.qwen_lm_stack(dev, synth.CONFIG, m["tl"], m["tf"], dtype)
    pstack = qtts.qwen_lm_stack(dev, synth.CONFIG, m["pl"], m["pf"], dtype)
    # the batched frames share the stacks; they run first and
    # are freed before the lms take ownership of the stacks
    batched = box = None
    if args.batch > 0 and dtype == "q8_0":
        batched = batched_frames(args, qtts, torch, tstack, th, pstack, ph, m, local_rank, rank, dist)
        if not args.only_batched and (args.talker_layers, args.pred_layers) == (28, 5):
            box = box_run(args, qtts, torch, tstack, th, pstack, ph, m, local_rank, rank, dist)
    if args.only_batched:
        # the configs[2] measurement alone (profiling runs)
        if rank == 0:
            print(json.dumps({"impl": "ours", "n_gpus": world, "batched": batched}), flush=True)
        for o in (th, ph):
            o.free()
        for st in (tstack, pstack):
            qtts.stack_destroy(st)
        dev.close()
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    prefill = None
    if args.prefill_steps > 0 and rank == 0 and (args.talker_layers, args.pred_layers) == (28, 5) or args.only_prefill:
        prefill = prefill_measure(args, qtts, torch, m, dev, rank)
    if args.only_prefill:
        # the configs[3] measurement alone (profiling runs)
        print(json.dumps({"impl": "ours", "prefill": prefill}), flush=True)
        for o in (th, ph):
            o.free()
        for st in (tstack, pstack):
            qtts.stack_destroy(st)
        dev.close()
        return
    tlm = qtts.QwenLm(tstack, th, max_pos)
    plm = qtts.QwenLm(pstack, ph, 32)
    tk = qtts.QwenTalker(tlm, plm, m["ce"], m["pe"], synth.CODEC_EOS)
    stream = torch.cuda.ExternalStream(tk.stream, device=torch.device("cuda", local_rank))

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def run_frames(n):
        """n frames on the device loop, restarting the utterance at eos."""
        done, restarts = 0, 0
        while done < n:
            got = tk.run(n - done).shape[0]
            done += got
            if done < n:
                tk.start(prompt, None, m["pad"])
                restarts += 1
        return restarts

    if args.trace_frame:
        # the phase trace alone (profiling runs)
        tk.start(prompt, None, m["pad"])
        print(json.dumps({"impl": "ours", "trace": trace_measure(qtts, tk)}), flush=True)
        for o in (tk, tlm, plm, th, ph):
            o.free()
        dev.close()
        return
    # warm-up
    tk.start(prompt, None, m["pad"])
    run_frames(W)
    # value: frames with everything resident
    tk.start(prompt, None, m["pad"])
    barrier()
    clocks = Clocks(local_rank) if rank == 0 else None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    restarts = run_frames(K)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop() if clocks else None
    talker_len0 = PROMPT_ROWS[dtype]
    # e2e: the public per-frame API, prompt from (pinned) host memory
    pin_prompt = torch.from_numpy(prompt).pin_memory().numpy()
    codes = np.zeros(16, np.int32)
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    f0.record(stream)
    tk.start(pin_prompt, None, m["pad"])
    n_e2e = 0
    while n_e2e < K:
        if tk.next_frame(codes):
            n_e2e += 1
        else:
            tk.start(pin_prompt, None, m["pad"])
    f1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = f0.elapsed_time(f1)
    wall_e2e = time.perf_counter() - w0
    # the same frames in sampling mode, the reference engine's default
    # (QwenSamplingFromConfig, talker.pas:203-230: temperature 0.9, top_k 50,
    # top_p 1 for both choosers); everything resident, device events
    tk.set_sampling(seed=SEED + rank)
    tk.start(prompt, None, m["pad"])
    run_frames(W)
    tk.start(prompt, None, m["pad"])
    barrier()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    restarts_s = run_frames(K)
    g1.record(stream)
    torch.cuda.synchronize()
    ms_s = g0.elapsed_time(g1)
    ms, ms_e2e, ms_s = max_over_ranks([ms, ms_e2e, ms_s], dist, "cpu")
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and (args.talker_layers, args.pred_layers) == (28, 5):
        # bounded CPU sample (~15 s of the oracle on all host cores), at N=1
        # only and in a process of its own
        cpu = cpu_sample(dtype)
    # the prompt of Start and the heads' load, on rank 0 (no timed collective
    # follows); a failure is recorded in the line, never fatal to it
    start_p = heads_l = codec = None
    if rank == 0 and (args.talker_layers, args.pred_layers) == (28, 5):
        try:
            start_p = start_prompt_measure(qtts, tk, dev, not args.no_cpu_baseline)
        except Exception as e:  # noqa: BLE001
            start_p = {"error": f"{type(e).__name__}: {e}"}
        try:
            heads_l = heads_load_measure(qtts, dev, m, not args.no_cpu_baseline)
        except Exception as e:  # noqa: BLE001
            heads_l = {"error": f"{type(e).__name__}: {e}"}
        try:
            codec = codec_measure(qtts, dev, not args.no_cpu_baseline)
        except Exception as e:  # noqa: BLE001
            codec = {"error": f"{type(e).__name__}: {e}"}
    if rank == 0:
        fps = job_value(world, K, ms)
        wb = weight_bytes_per_frame(dtype, args.talker_layers, args.pred_layers)
        kv = sum(kv_bytes_frame(talker_len0 + f, args.talker_layers, args.pred_layers) for f in range(K)) / K
        alg = wb + kv  # algorithmic bytes per launch (one frame)
        per_launch_s = ms / 1000.0 / K
        peaks = measured_peaks()
        peak = peaks["hbm_gbs"] if peaks else 6650.0
        achieved = alg / per_launch_s / 1e9
        traffic = ncu_traffic(dtype)
        prompt_bytes = prompt.size * 4 + 1024 * 4
        line = {
            "metric": metric_name(dtype), "value": fps, "unit": "frames/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": dtype_name(dtype),
            "data": "synthetic (seeded N(0,0.02) weights of the Qwen3-TTS talker/predictor architecture, N(0,1) prompt)",
            "config": config_dict(dtype, args),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if peaks else "fallback",
                         "kernel": "qtts::decode_kernel (frame mode)",
                         "algorithmic_bytes_per_launch": alg},
            "e2e": {"value": job_value(world, K, ms_e2e), "unit": "frames/s",
                    "h2d_bytes_per_step": prompt_bytes / K,
                    "d2h_bytes_per_step": 104 + (3072 * 4) / K,
                    "wall_s_rank0": wall_e2e, "includes": "qtts_talker_start (prompt upload + prefill) + K x qtts_talker_next_frame"},
            "gpu_launches": K + (2 * restarts),
            "clocks": clk,
            "cpu_baseline": cpu,
            "restarts_at_eos": restarts,
            "sampled": {"value": job_value(world, K, ms_s), "unit": "frames/s", "ms_per_frame": ms_s / K,
                        "mode": "sampling: temperature 0.9, top_k 50, top_p 1 for code 0 and the predictor "
                                "(qwen_tts defaults), seeded draws on the device", "restarts_at_eos": restarts_s},
            "batched": batched,
            "box": box,
            "prefill": prefill,
            "start_prompt": start_p,
            "heads_load": heads_l,
            "codec": codec,
            "weights_generation_s": m["gen_s"],
        }
        line["summary"] = summary(line)  # last key: it stays in a tail of the output
        print(json.dumps(line), flush=True)
    tk.free()
    tlm.free()
    plm.free()
    th.free()
    ph.free()
    dev.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=156)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--config", choices=["q8_0", "f32"], default="q8_0")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    # the bounded CPU sample of cpu_baseline, run by bench.py in a process of its own
    ap.add_argument("--cpu-sample", choices=["q8_0", "f32"], default=None, help=argparse.SUPPRESS)
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help=argparse.SUPPRESS)
    # configs[2] beside the bench line: B utterances decoded together (0: off)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--batch-steps", type=int, default=20)
    ap.add_argument("--box-utterances", type=int, default=1024, help="configs[4]: utterances of the box")
    ap.add_argument("--box-frames", type=int, default=BOX_FRAMES, help="configs[4]: frames per utterance")
    ap.add_argument("--batch-ctx", type=int, nargs=2, default=list(BATCH_CTX), metavar=("LO", "HI"))
    ap.add_argument("--only-batched", action="store_true", help="run the configs[2] measurement alone")
    # configs[3] beside the bench line: batched prefill steps (0: off)
    ap.add_argument("--prefill-steps", type=int, default=2)
    ap.add_argument("--only-prefill", action="store_true", help="run the configs[3] measurement alone")
    ap.add_argument("--only-codec", action="store_true", help="run the codec measurement alone")
    ap.add_argument("--trace-frame", action="store_true",
                    help="print the phase trace of one configs[1] frame alone (no batched/prefill legs: --batch 0 "
                         "--prefill-steps 0)")
    # smaller stacks for profiler captures only (the benchmark is 28 + 5)
    ap.add_argument("--talker-layers", type=int, default=28)
    ap.add_argument("--pred-layers", type=int, default=5)
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.cpu_sample:
        cpu_sample_main(args.cpu_sample, args.cpu_seconds)
    elif args.impl == "reference":
        reference_arm(args, rank)
    else:
        gpu_arm(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
