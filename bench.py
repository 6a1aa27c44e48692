#!/usr/bin/env python
"""Decode benchmark of the B200 quantized decode path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c4b1024] [--secondary c1]
                    [--impl ours|reference]

One step = one greedy decode pass over every sequence of the configuration's
batch.  The headline workload is the largest single-GPU configuration of the
benchmark (BASELINE configs[4] at its top sweep point): MiniMind3-64M shaped,
q8 weights, KV q8, SEQ 768, 1024 sequences per GPU, one seeded 512-token
prefix prefilled once, saved as MMKV1 and restored into every sequence slot,
then greedy decode from position 511.  The c1 configuration (q4, batch 1, KV
q16, SEQ 256, 128-token prompt) is measured after it and reported inside the
same JSON line (`secondary`).  Weights and prompts are seeded synthetic data
of the configurations' shapes, packed into MMCF containers byte-equal to the
reference packer's output (sha256 checked against tests/golden/golden.json).

`value` times K device-resident decode steps (inputs already in HBM, one CUDA
graph replay each, L2 flushed between steps); `e2e` times K steps through the
public API with host buffers (tokens and positions in, greedy tokens out).
For N > 1 every rank decodes its own 1024 sequences (weak scaling, no
data-path collective) and the time is the max over ranks.  `--impl reference`
times the reference arithmetic on the host cores instead: the CPU
restatement in oracle/ (the reference has no CPU engine; its GL path cannot
run here), on a bounded sample of the same configuration's sequences.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "vc4-gles2-inference_b200")
for _p in (PKG, os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "decode tokens/s per GPU and per box (1/2/4/8)"
KV_NAME = {16: "q16", 8: "q8"}
OPS = ["qkv", "attention", "wo", "ffn", None, "logits"]   # op 4 (w2) runs inside op 3
DTYPE = "int64 (exact integer dot products on dp4a / tcgen05 kind::i8), f32/f64 epilogues"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c4b1024")
    ap.add_argument("--secondary", default="c1",
                    help="comma-separated configurations measured after the headline one and reported inside "
                         "its JSON line ('' for none)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="bounded CPU baseline sample")
    ap.add_argument("--private-prefix", action="store_true",
                    help="restore the prefix into every slot's own rows instead of holding it once (shared)")
    ap.add_argument("--seq", type=int, default=0,
                    help="shorter KV cache (and prompt at most half of it) for small profiling captures")
    return ap.parse_args()


def model_path(cfg) -> str:
    """The configuration's container, written once per host and verified
    against the reference packer's sha256."""
    from vc4b200 import mmcf_writer
    d = os.path.join(tempfile.gettempdir(), "vc4b200_models")
    os.makedirs(d, exist_ok=True)
    key = cfg.extra.get("model", cfg.key)   # the c4 sweep shares one container
    path = os.path.join(d, "%s_%d.mmcf" % (key, cfg.seed))
    want = None
    try:
        with open(os.path.join(ROOT, "tests", "golden", "golden.json")) as f:
            want = json.load(f)["containers"].get(key, {}).get("sha256")
    except OSError:
        pass
    if os.path.exists(path):
        return path
    from vc4b200 import synth
    # the container of the configuration `key` names; a shortened session
    # (--seq) still decodes over the configuration's own container
    data = mmcf_writer.pack_config(dict(synth.CONFIGS, **synth.TINY_CONFIGS).get(key, cfg))
    if want and hashlib.sha256(data).hexdigest() != want:
        raise SystemExit("container for %s does not match the reference packer's bytes" % cfg.key)
    tmp = path + ".%d.tmp" % os.getpid()
    with open(tmp, "wb") as f:
        f.write(data)
    os.replace(tmp, path)
    return path


def sequence_ids(rank: int, batch: int) -> list:
    """The seeded sequences a rank decodes: rank r owns r*B .. r*B+B-1, so
    ranks never share a sequence and the job's work grows with the ranks."""
    return [rank * batch + b for b in range(batch)]


def workload_desc(cfg) -> str:
    s = cfg.shape
    if cfg.extra.get("prefix_restore"):
        how = ("one %d-token seeded prefix prefilled once, saved as MMKV1 and restored into every slot, "
               "then greedy decode" % cfg.prompt)
    else:
        how = "%d-token seeded prompt then greedy decode" % cfg.prompt
    return "%s: %s %s, batch %d, KV %s, SEQ %d, %s" % (cfg.key, s.name, cfg.quant, cfg.batch,
                                                       KV_NAME[cfg.kv_bits], cfg.seq, how)


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------

class Clocks:
    """SM clock and throttle reasons sampled while the timed region runs.

    NVML is polled from a thread every couple of milliseconds, so even a timed
    region of a few tens of milliseconds gets samples; nvidia-smi's 200 ms
    loop is the fallback when the NVML binding is missing."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device: int):
        self.sm, self.mx, self.reasons, self.p, self.nv = [], None, set(), None, None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = self._handle(pynvml, device)
            self.mx = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
            self.run = True
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return
        except Exception:
            self.nv = None
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.Q, "--format=csv,noheader,nounits",
                                       "-lms", "200", "-i", str(device)], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    @staticmethod
    def _handle(nv, device):
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            return nv.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
        except Exception:
            vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
            idx = int(vis.split(",")[device]) if vis and vis.split(",")[device].isdigit() else device
            return nv.nvmlDeviceGetHandleByIndex(idx)

    def _poll(self):
        nv = self.nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while self.run:
            try:
                self.sm.append(float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)))
                bits = get_reasons(self.h)
                for n, b in self.BITS.items():
                    if bits & b:
                        self.reasons.add(n)
            except Exception:
                pass
            time.sleep(0.002)

    def stop(self) -> dict:
        if self.nv is not None:
            self.run = False
            self.t.join(timeout=5)
            return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.mx,
                    "reasons": sorted(self.reasons), "samples": len(self.sm), "source": "nvml"}
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.flush()
        self.f.seek(0)
        rows = [l.split(",") for l in self.f.read().splitlines() if l.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for i, n in enumerate(names):
                    if r[5 + i].strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi"}


# ---------------------------------------------------------------------------
# distributed plumbing (one process per GPU, no data-path collective)
# ---------------------------------------------------------------------------

class Dist:
    """torchrun plumbing: rank/world from the environment, a process group
    used only for barriers and the max-over-ranks time (no data-path
    collective: every rank decodes its own sequences)."""

    def __init__(self, backend: str = "nccl", timeout_s: int = 120):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        self.pg = None
        if self.world > 1:
            import datetime
            import torch
            import torch.distributed as dist
            kw = {}
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                kw["device_id"] = torch.device("cuda", self.local)
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        return self._reduce(v, "max")

    def sum(self, v: float) -> float:
        return self._reduce(v, "sum")

    def _reduce(self, v: float, how: str) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device="cuda" if self.backend == "nccl" else "cpu")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX if how == "max" else self.pg.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# workload description (identical in both arms)
# ---------------------------------------------------------------------------

def config_of(cfg, world: int, private_prefix: bool = False) -> dict:
    restore = bool(cfg.extra.get("prefix_restore"))
    return {"workload": workload_desc(cfg), "batch_per_gpu": cfg.batch, "seq": cfg.seq, "quant": cfg.quant,
            "kv": KV_NAME[cfg.kv_bits], "prefix_restore": restore,
            "prefix_rows": ("each slot's own copy" if private_prefix else "held once per GPU, read by every slot")
                           if restore else None,
            "parallelism": ("dp%d (sequences sharded by rank)" % world) if cfg.batch > 1 else
                           ("dp%d replicas" % world),
            "l2": "flushed between timed steps (256 MiB write, then read back so no dirty line is left)"}


def decode_prompts(cfg, rank: int) -> list:
    """Each sequence's tokens up to and including the one its first decode
    step consumes.  A prefix-restore configuration shares one seeded prefix
    (prefilled once, restored into every slot) and parts at its last position
    with a distinct token per sequence."""
    from vc4b200 import synth
    ids = sequence_ids(rank, cfg.batch)
    if cfg.extra.get("prefix_restore"):
        prefix = synth.prompt_tokens(cfg, 0)
        return [prefix[:-1] + [(prefix[-1] + 97 * i) % cfg.shape.vocab] for i in ids]
    return [synth.prompt_tokens(cfg, i) for i in ids]


# ---------------------------------------------------------------------------
# the reference arithmetic on the host cores (oracle/)
# ---------------------------------------------------------------------------

class CpuDecode:
    """Greedy decode through the CPU restatement of the reference layer loop.
    The prompts are prefilled once (untimed, all host threads); a timed sample
    then decodes `seqs` of the configuration's sequences from their prompts'
    ends.  Sequences of one pass are independent, so the rate of a sample of
    them is the configuration's CPU tokens/s."""

    def __init__(self, cfg, path, seqs: int = 2):
        import oracle
        self.oracle = oracle
        self.cfg = cfg
        oracle.set_threads(os.cpu_count() or 1)
        self.om = oracle.Model(path)
        self.prompts = decode_prompts(cfg, 0)[:max(1, min(cfg.batch, seqs))]
        self.rows = []   # per sampled sequence: the prompt's KV rows of every layer
        shared = None
        for p in self.prompts:
            if cfg.extra.get("prefix_restore") and shared is not None:
                self.rows.append(shared)
                continue
            s = oracle.Session(self.om, cfg.kv_bits)
            for i, t in enumerate(p[:-1]):
                s.step(t, i, want_logits=False)
            r = [s.kv_rows(l, len(p) - 1) for l in range(self.om.info.layers)]
            s.close()
            self.rows.append(r)
            if cfg.extra.get("prefix_restore"):
                shared = r

    def rate(self, steps: int, seconds: float, threads: int) -> dict:
        self.oracle.set_threads(threads)
        done, total = 0, 0.0
        for p, rows in zip(self.prompts, self.rows):
            s = self.oracle.Session(self.om, self.cfg.kv_bits)
            for l, r in enumerate(rows):
                s.kv_write(l, len(p) - 1, r)
            tok, pos = p[-1], len(p) - 1
            t0 = time.perf_counter()
            for _ in range(steps):
                tok = self.oracle.argmax(s.step(tok, pos))
                pos += 1
                done += 1
                if pos >= self.cfg.seq or time.perf_counter() - t0 > seconds / len(self.prompts):
                    break
            total += time.perf_counter() - t0
            s.close()
        return {"value": done / total, "unit": "tokens/s", "cores": threads, "kind": "port",
                "sample": "%d greedy decode steps of %d of the configuration's sequences from position %d "
                          "(prompt prefilled untimed), oracle/ C restatement, OpenMP over matrix rows"
                          % (done, len(self.prompts), len(self.prompts[0]) - 1)}


def cpu_baseline(cfg, path, steps: int, seconds: float) -> dict:
    """All-core rate, plus the single-thread rate on a shorter sample."""
    cd = CpuDecode(cfg, path)
    allc = cd.rate(steps, seconds, os.cpu_count() or 1)
    one = cd.rate(steps, max(2.0, seconds / 3.0), 1)
    allc["single_thread"] = {"value": one["value"], "cores": 1, "sample": one["sample"]}
    return allc


def run_reference(args, cfg, dist):
    if dist.rank != 0:
        return
    path = model_path(args.model_cfg)
    threads = os.cpu_count() or 1
    cd = CpuDecode(cfg, path)
    # a step is one decode token of each sampled sequence
    r = cd.rate(max(1, args.steps + args.warmup), 10 * args.cpu_seconds, threads)
    line = {"metric": METRIC, "value": r["value"], "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000.0 / r["value"] * len(cd.prompts), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": DTYPE,
            "data": "synthetic (seeded weights and prompts of the configuration's shape)",
            "config": config_of(cfg, args.gpus, args.private_prefix),
            "impl": "reference", "cpu_baseline": r,
            "e2e": {"value": r["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# the B200 path
# ---------------------------------------------------------------------------

def peaks() -> tuple:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (measured)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6650 GB/s"


def measure(args, cfg, dist, full: bool = True) -> dict:
    """Decode throughput of one configuration on this rank's GPU: device-
    resident graph replays (`value`), then the public API with host buffers
    (`e2e`), then the live per-op replay probe for the roofline."""
    import ctypes as C

    import numpy as np
    import torch
    import vc4b200

    dev = dist.local
    torch.cuda.set_device(dev)
    path = model_path(cfg)
    gpu = vc4b200.GPU(dev)
    model = vc4b200.Model(gpu, path)
    B = cfg.batch
    sess = vc4b200.Session(model, slots=B, seq=cfg.seq, kv=KV_NAME[cfg.kv_bits])
    info = model.info
    prompts = decode_prompts(cfg, dist.rank)
    t0 = time.perf_counter()
    if cfg.extra.get("prefix_restore"):
        # one prefix prefilled once (batched prefill: its positions run as one
        # batch of the many-sequence path), saved as MMKV1 and restored into every slot
        prefix = prompts[0][:-1]
        sess.prefill(prefix, 0, slot=0, want_logits=False, batched=True)
        prefill_tok = len(prefix)
        prefill_only_s = time.perf_counter() - t0
        mmkv = os.path.join(tempfile.gettempdir(), "vc4b200_prefix_%d_%d.mmkv" % (os.getpid(), dist.rank))
        sess.save_prefix_cache(mmkv, prefix)
        if args.private_prefix:
            for b in range(1, B):
                sess.load_prefix_cache(mmkv, slot=b)
        else:
            # restored into every slot, the rows held once on the GPU
            sess.load_prefix_cache_shared(mmkv, list(range(B)))
        os.unlink(mmkv)
        if os.path.exists(mmkv + ".json"):
            os.unlink(mmkv + ".json")
    else:
        for b in range(B):
            sess.prefill(prompts[b][:-1], 0, slot=b, want_logits=False, batched=True)
        prefill_tok = sum(len(p) - 1 for p in prompts)
        prefill_only_s = time.perf_counter() - t0
    prefill_s = time.perf_counter() - t0
    prefill = {"tokens": prefill_tok, "s": prefill_only_s, "tokens_per_s": prefill_tok / prefill_only_s,
               "how": "vc4_prefill_batch (up to %d positions of a prompt per pass; the serial loop below 16 "
                      "positions), host wall clock with a synchronize per pass, first-call graph capture included"
                      % B}
    P = len(prompts[0])
    stream = torch.cuda.ExternalStream(sess.stream())
    d_slots = torch.arange(B, dtype=torch.int32, device="cuda")
    first = torch.tensor([p[-1] for p in prompts], dtype=torch.int32)
    d_tok = first.to("cuda")
    d_pos = torch.full((B,), P - 1, dtype=torch.int32, device="cuda")
    d_next = torch.zeros(B, dtype=torch.int32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def l2_flush(i):
        # evict L2 with a 256 MiB write, then read it back so the dirty lines
        # are written to DRAM here, not during the timed step
        flush.fill_(i & 0x7F)
        flush.view(torch.int32).max()
    torch.cuda.synchronize()
    pos_now = [P - 1]

    def step():
        if pos_now[0] >= cfg.seq:      # positions cycle within [P-1, seq)
            with torch.cuda.stream(stream):
                d_tok.copy_(first)
                d_pos.fill_(P - 1)
            pos_now[0] = P - 1
        sess.step_batch_device(B, d_slots.data_ptr(), d_tok.data_ptr(), d_pos.data_ptr(), d_next.data_ptr(), True)
        pos_now[0] += 1

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    l0, _ = sess.counters()
    clocks = Clocks(dev)
    dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            l2_flush(i)                           # L2 flush between steps (outside the events)
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    clk = clocks.stop()
    sess.check()
    l1, _ = sess.counters()
    ms = sum(a.elapsed_time(b) for a, b in ev)
    ms_max = dist.max(ms)
    tokens = dist.sum(B * args.steps)
    value = tokens / (ms_max / 1000.0)

    # e2e: the public API with host buffers, greedy tokens read back each step
    slots_h = np.arange(B, dtype=np.int32)
    tok_h = first.numpy().astype(np.int32)
    pos_h = np.full(B, P - 1, np.int32)
    torch.cuda.synchronize()
    e2e_s = 0.0
    dist.barrier()
    for i in range(args.steps):
        if pos_h[0] >= cfg.seq:
            tok_h, pos_h = first.numpy().astype(np.int32), np.full(B, P - 1, np.int32)
        l2_flush(i)
        torch.cuda.synchronize()
        t = time.perf_counter()
        if B == 1:
            nxt = np.array([sess.step_greedy(int(tok_h[0]), int(pos_h[0]))], np.int32)
        else:
            nxt = sess.step_batch(slots_h, tok_h, pos_h)
        e2e_s += time.perf_counter() - t
        tok_h, pos_h = nxt.astype(np.int32), pos_h + 1
    e2e_s = dist.max(e2e_s)
    e2e = {"value": tokens / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 12 * B, "d2h_bytes_per_step": 4 * B}

    # live per-op timing (replay probe, cold L2) for the roofline
    L = info.layers
    prof_pos = np.array([min(int(pos_h[0]), cfg.seq - 1)] * B, np.int32)
    op_ms, op_bytes = {}, {}
    P_ = vc4b200.engine._p
    for op in range(6):
        if OPS[op] is None:
            continue
        avg, byt = C.c_double(), C.c_double()
        rc = vc4b200.lib().vc4_profile_op(sess._h, op, L - 1, B, P_(slots_h), P_(tok_h), P_(prof_pos), 20, 1,
                                          C.byref(avg))
        if rc:
            raise RuntimeError(vc4b200.lib().vc4_last_error().decode())
        vc4b200.lib().vc4_op_bytes(sess._h, op, L - 1, B, P_(prof_pos), C.byref(byt))
        op_ms[OPS[op]] = avg.value
        op_bytes[OPS[op]] = byt.value
    per_step = {k: op_ms[k] * (1 if k == "logits" else L) for k in op_ms}
    dom = max(per_step, key=per_step.get)
    hbm, peak_src = peaks()
    achieved = op_bytes[dom] / (op_ms[dom] / 1000.0) / 1e9
    step_bytes = sum(op_bytes[k] * (1 if k == "logits" else L) for k in op_bytes)
    roofline = {"bound": "hbm", "kernel": KERNEL_OF[dom](B, info), "op": dom, "achieved": achieved, "peak": hbm,
                "unit": "GB/s", "frac": achieved / hbm, "limit": LIMIT_OF.get((dom, B >= 8), ""),
                # DRAM bytes need an ncu capture, which this run does not make
                "traffic": None, "peak_source": peak_src,
                "bytes_per_launch": op_bytes[dom], "ms_per_launch": op_ms[dom], "kv_position": int(prof_pos[0]),
                "step_bytes": step_bytes, "step_frac": step_bytes / (ms_max / args.steps / 1000.0) / 1e9 / hbm,
                "per_op_ms": op_ms, "per_op_bytes": op_bytes, "share_per_step": {
                    k: per_step[k] / (ms_max / args.steps) for k in per_step}}
    if full:
        roofline["matvec_batch1"] = matvec_roofline(dev, hbm)
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": dist.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": DTYPE,
            "data": "synthetic (seeded weights and prompts of the configuration's shape)",
            "config": config_of(cfg, dist.world, args.private_prefix), "prefill_s": prefill_s, "prefill": prefill,
            "roofline": roofline, "e2e": e2e, "clocks": clk, "gpu_launches": l1 - l0}
    sess.close()
    model.close()
    gpu.close()
    return line


# which kernel serves an op at a batch size (kernels.cu launch_* selection)
KERNEL_OF = {
    "qkv": lambda B, i: "k_tmm<qkv> (tcgen05)" if B >= 32 and i.wtype == 0 else "k_qkv" if B < 8 else "k_mm<qkv>",
    "attention": lambda B, i: "k_attn_b" if B * i.kv_heads * (1 if (i.heads // i.kv_heads) % 2 else
                                                                (i.heads // i.kv_heads) // 2) >= 32 else "k_attn",
    "wo": lambda B, i: "k_tmm<wo> (tcgen05)" if B >= 32 and i.wtype == 0 else "k_wo" if B < 8 else "k_mm<wo>",
    "ffn": lambda B, i: "k_tmm<w13>+k_tmm<w2> (tcgen05)" if B >= 32 and i.wtype == 0 else
                        "k_gate" if B < 8 else "k_mm<ffn>+k_mmdown",
    "logits": lambda B, i: "k_tmm<logits> (tcgen05)" if B >= 8 else "k_logits",
}


# What bounds the dominant kernel, from its ncu captures (the HBM fraction
# alone does not say it for these kernels)
LIMIT_OF = {
    ("attention", True): "instruction issue and per-CTA barrier chain, not DRAM: ncu issue active 47%, L2 hit rate "
                         "94% (the prefix held once is read from L2), see profiles/attn_b_c4b128.md",
    ("attention", False): "dependency latency: one launch moves well under 1 MB, see profiles/attn_c1.md",
    ("ffn", True): "epilogue instructions (exact row scalings, SwiGLU, w2 records), tensor pipe 5-9%, "
                   "see profiles/tmm_c4b1024.md",
}


def matvec_roofline(dev: int, hbm: float) -> dict:
    """Batch-1 matvec_s on large synthetic matrices (q8 of the c3 logits
    head's shape, 64 MiB of q4 and t3 weights; the configurations' other
    matrices are 0.3-5 MB, too small for one launch to reach HBM speed),
    cold L2 and warm, 100 launches each."""
    import ctypes as C
    import vc4b200
    out = {}
    for name, wt, rows, cols in (("q8", 0, 73448, 1024), ("q4", 1, 65536, 2048), ("t3", 2, 131072, 2048)):
        ent = {"rows": rows, "cols": cols}
        for mode, fl in (("cold", 1), ("warm", 0)):
            ms, byt, dig = C.c_double(), C.c_double(), C.c_uint64()
            rc = vc4b200.lib().vc4_matvec_probe(dev, wt, rows, cols, 0, 100, fl, C.byref(ms), C.byref(byt),
                                                C.byref(dig))
            if rc:
                raise RuntimeError(vc4b200.lib().vc4_last_error().decode())
            gbs = byt.value / (ms.value / 1000.0) / 1e9
            ent["bytes"] = byt.value
            ent[mode] = {"ms": ms.value, "gbs": gbs, "frac": gbs / hbm}
        out[name] = ent
    return out


def run_ours(args, cfg, dist):
    line = measure(args, cfg, dist, full=True)
    if dist.world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, model_path(cfg), args.steps, args.cpu_seconds)
    else:
        line["cpu_baseline"] = None
    if args.secondary:
        from vc4b200 import synth
        sec = []
        for key in args.secondary.split(","):
            c2 = synth.CONFIGS[key]
            l2 = measure(args, c2, dist, full=False)
            ent = {k: l2[k] for k in ("value", "ms_per_step", "e2e", "gpu_launches", "clocks", "prefill")}
            ent["config"] = l2["config"]
            ent["roofline"] = {k: l2["roofline"][k] for k in ("kernel", "op", "achieved", "frac", "step_frac",
                                                             "per_op_ms", "share_per_step")}
            if dist.world == 1 and not args.no_cpu_baseline:
                ent["cpu_baseline"] = cpu_baseline(c2, model_path(c2), args.steps, args.cpu_seconds / 2)
            sec.append(ent)
        line["secondary"] = sec
    if dist.rank == 0:
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    from vc4b200 import synth
    cfg = dict(synth.CONFIGS, **synth.TINY_CONFIGS)[args.config]
    args.model_cfg = cfg   # the container is always the configuration's own
    if args.seq:
        import dataclasses
        cfg = dataclasses.replace(cfg, seq=args.seq, prompt=min(cfg.prompt, args.seq // 2),
                                  extra=dict(cfg.extra, model=cfg.extra.get("model", cfg.key)))
    dist = Dist()
    try:
        if args.impl == "reference":
            run_reference(args, cfg, dist)
        else:
            run_ours(args, cfg, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
