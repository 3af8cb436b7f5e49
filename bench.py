"""Benchmark of the paged-KV hot path: one layer's KV append + paged decode.

Workload ("config 2"): Qwen3-8B heads (32 q / 8 KV,
head_dim 128), bf16, block_size 16, batch 256, every context 4096 tokens,
65,536-block KV pool with seeded-permuted block tables; the append writes the
256 new K/V rows, then decode attention reads 4 GiB of paged KV.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

With N > 1 (launched by torchrun, one process per GPU) the KV heads are
sharded N ways, as the engine's tensor parallelism does: rank r owns KV
heads [r*8/N, (r+1)*8/N) and their q heads, its own cache shard and the same
block tables. There is no collective on the data path; ranks meet only at the
timing barriers. `value` = algorithmic bytes of all ranks / max rank time.

`--impl reference` times the reference's own CPU implementation of the path —
the unmodified engine installed in baseline/_ref: KVCacheStore.forward_native
(nanovllm/layers/attention.py:69-85) and _paged_attention_reference
(tests/test_attention_backend.py:660-699) — on the full config 2 batch, with
all host threads, on rank 0 only.

The default line also carries sub-records measured after the headline on the
same GPU (N = 1 only), each with its own roofline: config 3's mixed step and
its prefill kernel, config 5 at block sizes 16 and 256, a 4 x 8192-token
causal prefill, and the plain KV append at 65,536 rows.
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
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))
from baseline import install_ref  # noqa: E402

# The engine this backend plugs into (nanovllm), installed unmodified into
# baseline/_ref, and the reference's test helpers the reference arm times.
ENGINE_INSTALLED = install_ref.add_to_path()
METRIC = "paged decode attn+KV-append HBM GB/s and tokens/s at 1/2/4/8 B200"
TOTAL_Q_HEADS, TOTAL_KV_HEADS, HEAD_DIM, BLOCK_SIZE = 32, 8, 128, 16
BATCH, CONTEXT = 256, 4096
SEED_LONG_PREFILL, SEED_APPEND = 2026 + 7, 2026 + 8
WORKLOAD = ("config2: Qwen3-8B decode step, one layer: KV append of 256 rows + paged GQA "
            "decode, B 256, ctx 4096, Hq 32 / Hkv 8, D 128, bs 16, bf16")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--cpu-sample-seqs", type=int, default=32,
                    help="sequences of the bounded CPU-baseline sample in the GPU arm")
    ap.add_argument("--no-subrecords", action="store_true",
                    help="skip the config 3 / config 5 / prefill / append sub-records")
    ap.add_argument("--batch", type=int, default=BATCH,
                    help="smaller batches are for profiler captures only")
    ap.add_argument("--workload", choices=("config2", "config3", "config4", "rope_append",
                                           "config5_bs16", "config5_bs256", "prefill_long",
                                           "append_64k"),
                    default="config2",
                    help="config3: mixed chunked prefill + decode (1 GPU), reports the "
                         "prefill kernel against the tensor roofline; rope_append: the "
                         "fused q/k-norm + RoPE + KV append kernel (1 GPU)")
    ap.add_argument("--kv-dtype", choices=("bf16", "fp8"), default="bf16",
                    help="fp8: the config 2 step over an FP8 E4M3 KV pool (scales 1.0); "
                         "bytes are counted at one byte per element")
    ap.add_argument("--comparator", choices=("none", "flashinfer"), default="none",
                    help="flashinfer: also time the library decode the reference engine calls "
                         "(BatchDecodeWithPagedKVCacheWrapper, configured as "
                         "FlashInferBackend does) on the same config 2 inputs; one extra line")
    ap.add_argument("--rope-tokens", type=int, default=16384,
                    help="tokens per rope_append step (a long prefill chunk)")
    return ap.parse_args()


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """SM clock, max clock, power and throttle reasons of the ranks' GPUs,
    sampled through NVML every millisecond on a background thread (ctypes
    releases the GIL during each call), so a timed region of a few
    milliseconds still holds several samples. Falls back to a 200 ms
    ``nvidia-smi`` loop where NVML cannot be loaded."""

    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices, period_s=0.001):
        self.gpus = list(gpu_indices)
        self.period = period_s
        self.samples = []  # (time, gpu, sm_mhz, sm_max_mhz, power_w, reasons)
        self.window = None
        self.source = None
        self._stop = threading.Event()
        self._thread = None
        self._proc = None

    def start(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            handles = [(g, pynvml.nvmlDeviceGetHandleByIndex(g)) for g in self.gpus]
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            max_sm = {g: pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
                      for g, h in handles}
        except Exception:  # no NVML: nvidia-smi at its 200 ms minimum
            self._start_smi()
            return
        self.source = f"NVML every {self.period * 1e3:g} ms"

        def loop():
            while not self._stop.is_set():
                now = time.time()
                for g, h in handles:
                    try:
                        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        bits = get_reasons(h)
                        power = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                    except Exception:
                        continue
                    reasons = [n for n, b in self.REASON_BITS.items() if bits & b]
                    self.samples.append((now, g, float(sm), float(max_sm[g]), power, reasons))
                self._stop.wait(self.period)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()

    def _start_smi(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self._proc = None
            return
        self.source = "nvidia-smi every 200 ms"
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

        def read():
            for line in self._proc.stdout:
                r = [c.strip() for c in line.split(",")]
                if len(r) < 9 or not r[0].isdigit() or int(r[0]) not in self.gpus:
                    continue
                try:
                    sm, smax = float(r[1]), float(r[2])
                except ValueError:
                    continue
                power = float(r[3]) if r[3].replace(".", "").isdigit() else 0.0
                reasons = [n for n, v in zip(names, r[5:9]) if v.lower() == "active"]
                self.samples.append((time.time(), int(r[0]), sm, smax, power, reasons))

        self._thread = threading.Thread(target=read, daemon=True)
        self._thread.start()

    def mark(self, t0, t1):
        self.window = (t0, t1)

    def stop(self):
        self._stop.set()
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self):
        rows = list(self.samples)
        note = "during the timed region"
        if self.window is not None:
            t0, t1 = self.window
            inside = [r for r in rows if t0 <= r[0] <= t1]
            if inside:
                rows = inside
            else:
                note = "around the timed region (no sample inside it)"
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "source": self.source}
        sm = [r[2] for r in rows]
        return {"sm_mhz": statistics.median(sm), "sm_min_mhz": min(sm),
                "sm_max_mhz": max(r[3] for r in rows),
                "power_w_max": round(max(r[4] for r in rows), 1),
                "reasons": sorted({n for r in rows for n in r[5]}),
                "samples": len(rows), "when": note, "source": self.source}


def physical_gpu_indices(world):
    """nvidia-smi indices of the GPUs the ranks use (CUDA_VISIBLE_DEVICES aware)."""
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v.strip() for v in visible.split(",") if v.strip()]
    if ids and all(v.isdigit() for v in ids):
        return [int(v) for v in ids[:world]]
    return list(range(world))


# ---------------------------------------------------------------- workload --
def make_shard(rank, world, device, batch=BATCH):
    import workloads

    if TOTAL_KV_HEADS % world:
        raise SystemExit(f"--gpus must divide {TOTAL_KV_HEADS} (KV heads are sharded)")
    return workloads.config2(device=device, seed=workloads.SEED_BASE + 2 + 1000 * rank,
                             num_kv_heads=TOTAL_KV_HEADS // world,
                             num_q_heads=TOTAL_Q_HEADS // world, batch=batch)


def peaks():
    try:
        data = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
        return float(data["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def committed_traffic():
    """Per-launch DRAM bytes of the decode kernel from the committed ncu
    summary (profiles/decode_config2_traffic.json), or None."""
    path = REPO / "profiles" / "decode_config2_traffic.json"
    try:
        data = json.loads(path.read_text())
        return int(data["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError):
        return None


# ------------------------------------------------------------ CPU baseline --
def reference_cpu_path():
    """The reference's own CPU implementation of the path, from the unmodified
    engine installed in baseline/_ref: ``KVCacheStore.forward_native``
    (nanovllm/layers/attention.py:69-85, selected by platform "cpu") and the
    fp32 ``_paged_attention_reference`` of its test suite
    (tests/test_attention_backend.py:660-699). None where it is not installed."""
    from baseline import install_ref

    if not install_ref.add_to_path():
        return None
    from nanovllm.layers.attention import KVCacheStore
    from nanovllm.layers.custom_op import CustomOpConfig
    from test_attention_backend import _paged_attention_reference

    return KVCacheStore(CustomOpConfig(platform="cpu")), _paged_attention_reference


def cpu_sample(num_seqs, seed=7):
    """A CPU-resident config 2 batch of `num_seqs` sequences of 4096 tokens
    (all 256 = the full workload), same heads, dtype and layout."""
    import workloads

    return workloads.config2(device="cpu", seed=seed, batch=num_seqs, ctx=CONTEXT)


def reference_csr(w):
    """kv_indptr / page_indices from the dense tables, as the engine's
    FlashInferBackend.build_metadata builds them for trusted metadata
    (attention_backend.py:700-713); the reference attention takes this CSR."""
    offsets = [0]
    for count in w.block_counts:
        offsets.append(offsets[-1] + count)
    kv_indptr = torch.tensor(offsets, dtype=torch.int32)
    page_indices = torch.cat(tuple(w.block_tables[row, :count]
                                   for row, count in enumerate(w.block_counts))).contiguous()
    return kv_indptr, page_indices


def make_reference_step(w):
    """One step of the reference's CPU path over workload `w`: the append of
    the new rows, then attention of every sequence. Returns (step, kind)."""
    path = reference_cpu_path()
    if path is not None:
        store, attend = path
        kv_indptr, page_indices = reference_csr(w)
        q_lens = tuple([1] * w.num_seqs)
        kv_lens = tuple(w.extra["seq_lens_host"])

        def step():
            store(w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping)
            attend(w.q, w.k_cache, w.v_cache, kv_indptr, page_indices, q_lens, kv_lens)

        return step, "reference"
    return (lambda: time_oracle(w, os.cpu_count() or 1)), "port"


def time_oracle(w, threads):
    """The oracle port of the same two steps (used only where the reference
    engine is not installed): sequences split across `threads` host threads."""
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np

    sys.path.insert(0, str(REPO))
    import oracle

    def bits(t):
        t = t.contiguous()
        return t.view(torch.int16).numpy().view(np.uint16)

    key, value = bits(w.key), bits(w.value)
    k_cache, v_cache = bits(w.k_cache), bits(w.v_cache)
    q = bits(w.q)
    tables = w.block_tables.numpy()
    lens = w.seq_lens.numpy()
    slots = w.slot_mapping.numpy()
    B = lens.size
    chunks = [list(range(i, B, threads)) for i in range(min(threads, B))]

    def run(ids):
        idx = np.array(ids)
        indptr, pages = oracle.block_tables_to_csr(tables[idx], lens[idx], w.block_size)
        return oracle.paged_attention(q[idx], k_cache, v_cache, indptr, pages, [1] * len(ids),
                                      lens[idx].tolist(), dtype="bfloat16")

    oracle.kv_append(key, value, k_cache, v_cache, slots)
    with ThreadPoolExecutor(max_workers=len(chunks)) as pool:
        list(pool.map(run, chunks))


def cpu_baseline_leg(sample_seqs):
    """The reference's CPU path on a bounded sample (about 10 s of CPU work)."""
    torch.set_num_threads(os.cpu_count() or 1)
    w = cpu_sample(sample_seqs)
    bytes_per_run = w.kv_bytes_read() + w.append_bytes()
    step, kind = make_reference_step(w)
    step()  # warm
    runs, elapsed = 0, 0.0
    while elapsed < 10.0 and runs < 500:
        t0 = time.perf_counter()
        step()
        elapsed += time.perf_counter() - t0
        runs += 1
    gbs = bytes_per_run * runs / elapsed / 1e9
    what = ("the reference's KVCacheStore.forward_native + _paged_attention_reference"
            if kind == "reference" else "the numpy oracle port")
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": kind,
            "sample": f"{sample_seqs} of the 256 sequences (ctx 4096, 8 KV heads), append + "
                      f"decode through {what}, {runs} runs in {elapsed:.1f} s"}


def run_reference(args, rank):
    """The reference arm: the reference's own CPU path on the FULL config 2
    batch (256 sequences x 4096 tokens) every step, all host threads."""
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    w = cpu_sample(BATCH, seed=7)
    bytes_per_step = w.kv_bytes_read() + w.append_bytes()
    step, kind = make_reference_step(w)
    for _ in range(args.warmup):
        step()
    total = 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        total += time.perf_counter() - t0
    gbs = bytes_per_step * args.steps / total / 1e9
    what = ("KVCacheStore.forward_native + _paged_attention_reference from the unmodified "
            "engine (baseline/_ref)" if kind == "reference" else "numpy oracle port")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": BATCH, "seq_len": CONTEXT,
                   "parallelism": "host CPU, rank 0 only"},
        "tokens_per_s": round(BATCH * args.steps / total, 2),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s",
                         "cores": torch.get_num_threads(), "kind": kind,
                         "sample": f"the full batch (256 sequences) every step, {what}"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- ours --
def run_ours(args, rank, world, local_rank):
    from my_vllm_b200 import B200PagedBackend, ops

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
    w = make_shard(rank, world, device, args.batch)
    fp8 = args.kv_dtype == "fp8"
    if fp8:
        import workloads

        w.k_cache = workloads.to_fp8_cache(w.k_cache, 1.0)
        w.v_cache = workloads.to_fp8_cache(w.v_cache, 1.0)
        torch.cuda.empty_cache()
        ops.register_kv_scales(w.k_cache, w.v_cache,
                               torch.ones(1, device=device), torch.ones(1, device=device))
    backend = B200PagedBackend(w.num_q_heads, w.num_kv_heads, HEAD_DIM, BLOCK_SIZE,
                               torch.bfloat16,
                               kv_cache_dtype=torch.float8_e4m3fn if fp8 else None)
    common = w.common_metadata()
    plan = backend.build_plan(common)
    kv_bytes = w.kv_bytes_read()
    app_bytes = w.append_bytes()
    step_bytes = kv_bytes + app_bytes
    n_parts = plan.metadata.decode_plan.num_parts
    launches_per_step = 2 + (1 if n_parts > 1 else 0)
    stream = torch.cuda.current_stream(device)

    def step():
        ops.store_kvcache(w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping)
        return backend.forward(w.q, w.key, w.value, w.k_cache, w.v_cache, plan)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    sampler = None
    if rank == 0 and not args.no_clocks:
        sampler = ClockSampler(physical_gpu_indices(world))
        sampler.start()

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(device)

    # The engine replays a decode step as a CUDA graph (full-decode graph
    # path), so the device-timed loop does too: the K timed steps (append +
    # attention each, in order) are captured as ONE graph, so host launch cost
    # and the gaps between separately launched graphs stay off the GPU
    # timeline, which matters at 8 GPUs where a step is ~0.1 ms. The decode
    # launch is then timed on its own, replayed as a graph of one launch with
    # events around each replay, for the roofline.
    timed_state = backend.create_full_decode_graph_state(
        w.num_seqs, w.num_seqs * w.block_tables.size(1), device)
    backend.plan_full_decode_graph(timed_state, plan)
    n_parts = timed_state.decode_plan.num_parts  # the replayed decode's split
    launches_per_step = 2 + (1 if n_parts > 1 else 0)

    def append():
        ops.store_kvcache(w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping)

    def attend():
        backend.forward(w.q, w.key, w.value, w.k_cache, w.v_cache, plan)

    def capture(body):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            body()
        return g

    backend.activate_full_decode_graph(timed_state)
    try:
        append()
        attend()
        torch.cuda.synchronize(device)
        steps_graph = capture(lambda: [(append(), attend()) for _ in range(args.steps)])
        decode_graph = capture(attend)
    finally:
        backend.deactivate_full_decode_graph()
    for _ in range(max(3, args.warmup)):
        append()
        decode_graph.replay()
    steps_graph.replay()  # one untimed pass of the timed graph itself
    torch.cuda.synchronize(device)

    # ---- device-timed region: the K steps as one graph replay ----
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(device)
    wall0 = time.time()
    t_start.record(stream)
    steps_graph.replay()
    t_end.record(stream)
    torch.cuda.synchronize(device)
    wall1 = time.time()
    barrier()
    elapsed_ms = max_over_ranks(t_start.elapsed_time(t_end))

    # ---- the decode launch alone (per-launch events), for the roofline ----
    dec_start = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    dec_end = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for i in range(args.steps):
        dec_start[i].record(stream)
        decode_graph.replay()
        dec_end[i].record(stream)
    torch.cuda.synchronize(device)
    decode_ms = sum(a.elapsed_time(b) for a, b in zip(dec_start, dec_end)) / args.steps
    decode_ms_max = max_over_ranks(decode_ms)
    backend.check_status()

    # ---- end to end through the public API with host buffers ----
    # The engine runs a pure-decode step as a full-decode CUDA Graph
    # (ModelRunner.run_model -> build_plan -> plan_full_decode_graph -> replay,
    # model_runner.py:496-518 and 676-766). Each step here: one packed
    # host->device copy of that step's inputs from pinned memory, build_plan,
    # plan_full_decode_graph, a replay of the captured append + attention, and a
    # device->host copy of the output. Two staging slots let the copies of
    # neighbouring steps overlap this step's kernels on two copy streams; the
    # timed region ends only after the last output has landed on the host.
    layout = [("q", w.q), ("key", w.key), ("value", w.value), ("slot_mapping", w.slot_mapping),
              ("block_tables", w.block_tables), ("seq_lens", w.seq_lens),
              ("query_start_loc", w.query_start_loc)]
    offsets, total = {}, 0
    for name, t in layout:
        offsets[name] = total
        total += (t.numel() * t.element_size() + 255) // 256 * 256

    def views(buf):
        out = {}
        for name, t in layout:
            n = t.numel() * t.element_size()
            out[name] = buf[offsets[name]: offsets[name] + n].view(t.dtype).view(t.shape)
        return out

    host_packed = torch.empty(total, dtype=torch.uint8, pin_memory=True)
    for name, t in layout:
        views(host_packed)[name].copy_(t)
    staging = [torch.empty(total, dtype=torch.uint8, device=device) for _ in range(2)]
    sv = [views(buf) for buf in staging]
    for b in range(2):
        staging[b].copy_(host_packed)
    commons = [type(common)(**{**common.__dict__, "query_start_loc": sv[b]["query_start_loc"],
                               "seq_lens": sv[b]["seq_lens"], "slot_mapping": sv[b]["slot_mapping"],
                               "block_tables": sv[b]["block_tables"]}) for b in range(2)]
    width = w.block_tables.size(1)
    states = [backend.create_full_decode_graph_state(w.num_seqs, w.num_seqs * width, device)
              for _ in range(2)]
    out_dev = [torch.empty_like(w.q) for _ in range(2)]
    out_host = [torch.empty(w.q.shape, dtype=w.q.dtype, pin_memory=True) for _ in range(2)]
    graphs = []
    for b in range(2):
        plan_b = backend.build_plan(commons[b])
        backend.plan_full_decode_graph(states[b], plan_b)
        backend.activate_full_decode_graph(states[b])
        try:
            def body(b=b, plan_b=plan_b):
                d = sv[b]
                ops.store_kvcache(d["key"], d["value"], w.k_cache, w.v_cache, d["slot_mapping"])
                o = backend.forward(d["q"], d["key"], d["value"], w.k_cache, w.v_cache, plan_b)
                out_dev[b].copy_(o)

            body()
            torch.cuda.synchronize(device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                body()
            graphs.append(graph)
        finally:
            backend.deactivate_full_decode_graph()
    torch.cuda.synchronize(device)
    h2d = total
    d2h = out_host[0].numel() * out_host[0].element_size()
    h2d_stream = torch.cuda.Stream(device)
    d2h_stream = torch.cuda.Stream(device)
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    compute_done = [torch.cuda.Event() for _ in range(2)]
    d2h_done = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        b = i % 2
        h2d_stream.wait_event(compute_done[b])  # slot b's previous step has consumed it
        with torch.cuda.stream(h2d_stream):
            staging[b].copy_(host_packed, non_blocking=True)
            h2d_done[b].record(h2d_stream)
        stream.wait_event(h2d_done[b])
        stream.wait_event(d2h_done[b])
        step_plan = backend.build_plan(commons[b])
        backend.plan_full_decode_graph(states[b], step_plan)
        graphs[b].replay()
        compute_done[b].record(stream)
        d2h_stream.wait_event(compute_done[b])
        with torch.cuda.stream(d2h_stream):
            out_host[b].copy_(out_dev[b], non_blocking=True)
            d2h_done[b].record(d2h_stream)

    for i in range(4):
        e2e_step(i)
    torch.cuda.synchronize(device)
    e2e_steps = max(1, min(args.steps, 100))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(device)
    e0.record(stream)
    h2d_stream.wait_stream(stream)  # no copy of the timed steps starts before e0
    for i in range(e2e_steps):
        e2e_step(i)
    stream.wait_event(d2h_done[(e2e_steps - 1) % 2])
    e1.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)

    if sampler is not None:
        sampler.mark(wall0, wall1)
        sampler.stop()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not fp8:
        cpu = cpu_baseline_leg(args.cpu_sample_seqs)

    graphs.clear()  # release the captured graphs before tearing the process group down
    del steps_graph, decode_graph
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    extra = {}
    if world == 1 and not fp8 and not args.no_subrecords and args.batch == BATCH:
        extra = subrecords(device, min(args.steps, 50), args.warmup)

    ms_per_step = elapsed_ms / args.steps
    total_bytes = step_bytes * world
    peak, peak_kind = peaks()
    achieved = kv_bytes * world / (decode_ms_max * 1e-3) / 1e9  # all ranks' decode bytes
    per_gpu_achieved = kv_bytes / (decode_ms * 1e-3) / 1e9
    traffic = committed_traffic() if world == 1 and not fp8 else None
    line = {
        "metric": METRIC,
        "value": round(total_bytes / (ms_per_step * 1e-3) / 1e9, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(3, args.warmup),
        "ms_per_step": round(ms_per_step, 5),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16 (KV cache fp8-e4m3)" if fp8 else "bf16",
        "data": "synthetic",
        "config": {
            "workload": WORKLOAD + (", KV pool FP8 E4M3 (1 byte per element)" if fp8 else ""),
            "global_batch": args.batch,
            "seq_len": CONTEXT,
            "parallelism": f"kv-head shards x{world} (tp{world}), no data-path collective",
            "l2": "inputs larger than L2: 4 GiB of paged KV per step across the ranks",
            "decode_split": n_parts,
            "timed_loop": "the K steps (append + attention each) captured as one CUDA graph "
                          "and replayed once (full-decode graph path); the decode launch timed "
                          "separately for the roofline",
        },
        "tokens_per_s": round(args.batch / (ms_per_step * 1e-3), 1),
        "bytes_per_step": total_bytes,
        "roofline": {
            "bound": "hbm",
            "kernel": "paged_decode_kernel",
            "achieved": round(per_gpu_achieved, 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(per_gpu_achieved / peak, 4),
            "peak_source": f"{peak_kind} HBM copy bandwidth (MEASURED_PEAKS.json hbm_gbs)",
            "frac_of_8tbs_nominal": round(per_gpu_achieved / 8000.0, 4),
            "algorithmic_bytes_per_launch": kv_bytes,
            "launch_ms": round(decode_ms, 5),
            "traffic": traffic,
            "all_ranks_achieved": round(achieved, 1),
        },
        "e2e": {
            "value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 2),
            "unit": "GB/s",
            "ms_per_step": round(e2e_ms, 5),
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "api": "engine full-decode CUDA Graph step: packed H2D from pinned memory, "
                   "B200PagedBackend.build_plan + plan_full_decode_graph, graph replay of "
                   "ops.store_kvcache + B200PagedBackend.forward, D2H of the output; copies of "
                   "neighbouring steps overlapped on two copy streams",
        },
        "gpu_launches": launches_per_step * args.steps,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if sampler is not None:
        line["clocks"] = sampler.summary()
    line.update(extra)
    print(json.dumps(line), flush=True)


def visible_pairs(q_len, kv_len):
    """Query-key pairs a causal chunk of q_len queries on kv_len keys sees."""
    return q_len * (kv_len - q_len) + q_len * (q_len + 1) // 2


def tensor_peak():
    try:
        peaks_data = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
        return float(peaks_data["bf16_tflops"]), "measured burst cuBLAS bf16 (MEASURED_PEAKS.json)"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def event_ms(fn, steps, warmup, stream, between=None):
    """Average device time of `fn` per call (CUDA events on `stream` around
    every call); `between` runs untimed before each call (an L2 flush)."""
    for _ in range(max(3, warmup)):
        if between is not None:
            between()
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for a, b in ev:
        if between is not None:
            between()
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in ev) / steps


def measure_config3(device, steps, warmup, fp8=False):
    """Config 3 (mixed chunked prefill + decode) on one GPU: the step is the
    engine's MIXED route — append 2172 rows, prefill rows [0, 2048) on the
    tcgen05 kernel, decode rows [2048, 2172) — and each kernel timed on its own
    (back to back, so the decode's 2 GB stream separates prefill launches)."""
    import workloads
    from my_vllm_b200 import B200PagedBackend, ops

    w = workloads.config3(device=device)
    scales = {}
    if fp8:
        w.k_cache = workloads.to_fp8_cache(w.k_cache, 1.0)
        w.v_cache = workloads.to_fp8_cache(w.v_cache, 1.0)
        ones = torch.ones(1, device=device)
        ops.register_kv_scales(w.k_cache, w.v_cache, ones, ones)
        scales = {"k_scale": ones, "v_scale": ones}
    backend = B200PagedBackend(w.num_q_heads, w.num_kv_heads, HEAD_DIM, BLOCK_SIZE,
                               torch.bfloat16,
                               kv_cache_dtype=torch.float8_e4m3fn if fp8 else None)
    common = w.common_metadata()
    plan = backend.build_plan(common)
    md = plan.metadata
    nP, P = common.num_prefill_seqs, common.num_prefill_tokens
    out = torch.empty_like(w.q)
    qsl, lens = w.extra["qsl_host"], w.extra["seq_lens_host"]
    flops = sum(4 * w.num_q_heads * HEAD_DIM * visible_pairs(qsl[i + 1] - qsl[i], lens[i])
                for i in range(nP))
    es = w.k_cache.element_size()
    prefill_kv_bytes = sum(lens[:nP]) * w.num_kv_heads * HEAD_DIM * es * 2
    decode_kv_bytes = sum(lens[nP:]) * w.num_kv_heads * HEAD_DIM * es * 2
    step_bytes = prefill_kv_bytes + decode_kv_bytes + w.append_bytes()
    stream = torch.cuda.current_stream(device)

    prefill_ws = backend._prefill_workspace_for(device)  # the backend's split-KV workspace

    def prefill():
        ops.paged_prefill(w.q[:P], w.k_cache, w.v_cache, md.block_tables[:nP],
                          md.seq_lens[:nP], md.query_start_loc[: nP + 1], out[:P],
                          common.max_q_len, backend.softmax_scale, num_seqs=nP,
                          workspace=prefill_ws, **scales)

    def decode():
        ops.paged_decode(w.q[P:], w.k_cache, w.v_cache, md.block_tables[nP:],
                         md.seq_lens[nP:], out[P:], md.decode_plan, backend.softmax_scale,
                         backend._workspace, **scales)

    def step():  # the engine's MIXED route: decode || prefill on two streams
        ops.store_kvcache(w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping)
        backend.forward(w.q, w.key, w.value, w.k_cache, w.v_cache, plan)

    for _ in range(max(3, warmup)):
        step()
    torch.cuda.synchronize()
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(steps):
        step()
    s1.record(stream)
    torch.cuda.synchronize()
    step_ms = s0.elapsed_time(s1) / steps

    # per-kernel rooflines: the same kernels launched back to back on one stream
    for _ in range(max(3, warmup)):
        ops.store_kvcache(w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping)
        prefill()
        decode()
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(steps):
        ops.store_kvcache(w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping)
        ev[i][0].record(stream)
        prefill()
        ev[i][1].record(stream)
        ev[i][2].record(stream)
        decode()
        ev[i][3].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    backend.check_status()
    serial_ms = t0.elapsed_time(t1) / steps
    pre_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / steps
    dec_ms = sum(e[2].elapsed_time(e[3]) for e in ev) / steps
    tflops_peak, src = tensor_peak()
    hbm, hbm_src = peaks()
    pre_tf = flops / (pre_ms * 1e-3) / 1e12
    dec_gbs = decode_kv_bytes / (dec_ms * 1e-3) / 1e9
    return {
        "workload": "config3: 4 x 512-token prefill chunks on shared prefix hits "
                    "0/512/1024/2048 + 124 decode rows ctx U[128, 8192], Qwen3-8B heads, bs 16; "
                    "append 2172 rows" + ("; KV pool FP8 E4M3" if fp8 else ""),
        "value": round(step_bytes / (step_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
        "ms_per_step": round(step_ms, 5), "serial_ms_per_step": round(serial_ms, 5),
        "steps": steps,
        "roofline": {"bound": "hbm", "kernel": "paged_decode_kernel",
                     "achieved": round(dec_gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(dec_gbs / hbm, 4), "peak_source": f"{hbm_src} hbm_gbs",
                     "launch_ms": round(dec_ms, 5),
                     "algorithmic_bytes_per_launch": decode_kv_bytes},
        "roofline_prefill": {"bound": "tensor", "kernel": "paged_prefill_tc_kernel",
                             "achieved": round(pre_tf, 1), "peak": tflops_peak,
                             "unit": "TFLOP/s", "frac": round(pre_tf / tflops_peak, 4),
                             "peak_source": src, "launch_ms": round(pre_ms, 5),
                             "algorithmic_flops_per_launch": flops},
        "gpu_launches": 3 * steps,
    }


def measure_config5(device, block_size, steps, warmup):
    """Config 5: long-context split-KV decode, B 32 x 32768 tokens (4 GiB of
    KV per step), Qwen3-8B heads, at block size 16 or 256."""
    import workloads
    from my_vllm_b200 import B200PagedBackend, ops

    w = workloads.config5(device=device, block_size=block_size)
    backend = B200PagedBackend(w.num_q_heads, w.num_kv_heads, HEAD_DIM, block_size,
                               torch.bfloat16)
    plan = backend.build_plan(w.common_metadata())
    stream = torch.cuda.current_stream(device)
    ops.store_kvcache(w.key, w.value, w.k_cache, w.v_cache, w.slot_mapping)
    ms = event_ms(lambda: backend.forward(w.q, w.key, w.value, w.k_cache, w.v_cache, plan),
                  steps, warmup, stream)
    backend.check_status()
    hbm, src = peaks()
    kv = w.kv_bytes_read()
    gbs = kv / (ms * 1e-3) / 1e9
    parts = plan.metadata.decode_plan.num_parts
    return {
        "workload": f"config5: B 32, ctx 32768, Hq 32 / Hkv 8, D 128, bs {block_size}, bf16, "
                    "split-KV decode + reduce",
        "value": round(gbs, 1), "unit": "GB/s", "ms_per_step": round(ms, 5), "steps": steps,
        "decode_split": parts,
        "roofline": {"bound": "hbm", "kernel": "paged_decode_kernel + decode_reduce_kernel",
                     "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gbs / hbm, 4), "peak_source": f"{src} hbm_gbs",
                     "launch_ms": round(ms, 5), "algorithmic_bytes_per_launch": kv},
        "gpu_launches": (2 if parts > 1 else 1) * steps,
    }


def measure_prefill_long(device, steps, warmup, seqs=4, tokens=8192):
    """Steady-state prefill rate: `seqs` fresh causal prefills of `tokens`
    tokens each (no prefix), Qwen3-8B heads — long enough that per-CTA
    set-up and the last wave's tail are small next to the steady state."""
    import workloads
    from my_vllm_b200 import ops

    w = workloads.small_case([tokens] * seqs, [tokens] * seqs, seqs, Hq=32, Hkv=8,
                             device=device, seed=SEED_LONG_PREFILL)
    out = torch.empty_like(w.q)
    stream = torch.cuda.current_stream(device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    ws = torch.zeros(ops.prefill_workspace_bytes(), dtype=torch.uint8, device=device)
    ms = event_ms(lambda: ops.paged_prefill(w.q, w.k_cache, w.v_cache, w.block_tables,
                                            w.seq_lens, w.query_start_loc, out, tokens,
                                            HEAD_DIM ** -0.5, status=status, workspace=ws),
                  steps, warmup, stream)
    if int(status.item()):
        raise RuntimeError(f"prefill reported status {int(status.item())}")
    flops = seqs * 4 * 32 * HEAD_DIM * visible_pairs(tokens, tokens)
    tf = flops / (ms * 1e-3) / 1e12
    peak, src = tensor_peak()
    return {
        "workload": f"prefill_long: {seqs} x {tokens}-token causal prefill, no prefix, Hq 32 / "
                    "Hkv 8, D 128, bs 16, bf16",
        "value": round(tf, 1), "unit": "TFLOP/s", "ms_per_step": round(ms, 5), "steps": steps,
        "roofline": {"bound": "tensor", "kernel": "paged_prefill_tc_kernel",
                     "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(tf / peak, 4), "peak_source": src,
                     "launch_ms": round(ms, 5), "algorithmic_flops_per_launch": flops},
        "gpu_launches": steps,
    }


def measure_append(device, steps, warmup, rows=65536):
    """The plain KV append (store_kvcache) at a size where it is not
    launch-bound: `rows` new K/V rows of Qwen3-8B (8 KV heads x 128, bf16)
    scattered to random slots of a pool twice that size. Algorithmic bytes:
    read the K and V rows, write them into the cache (2 x 2 x rows x 2 KiB)."""
    from my_vllm_b200 import ops

    g = torch.Generator(device=device).manual_seed(SEED_APPEND)
    key = torch.randn(rows, TOTAL_KV_HEADS, HEAD_DIM, generator=g, device=device).bfloat16()
    value = torch.randn_like(key)
    blocks = 2 * rows // BLOCK_SIZE
    k_cache = torch.zeros(blocks, BLOCK_SIZE, TOTAL_KV_HEADS, HEAD_DIM, dtype=torch.bfloat16,
                          device=device)
    v_cache = torch.zeros_like(k_cache)
    slots = torch.randperm(blocks * BLOCK_SIZE, generator=g, device=device)[:rows].int()
    stream = torch.cuda.current_stream(device)
    ms = event_ms(lambda: ops.store_kvcache(key, value, k_cache, v_cache, slots), steps,
                  warmup, stream)
    row_bytes = TOTAL_KV_HEADS * HEAD_DIM * 2
    alg = 2 * 2 * rows * row_bytes  # K and V, read + write
    gbs = alg / (ms * 1e-3) / 1e9
    hbm, src = peaks()
    return {
        "workload": f"append_64k: {rows} K/V rows (8 KV heads x 128, bf16) to random slots of a "
                    f"{blocks}-block pool",
        "value": round(gbs, 1), "unit": "GB/s", "ms_per_step": round(ms, 5), "steps": steps,
        "l2": f"{alg / 1e6:.0f} MB per launch (> 126 MB L2)",
        "roofline": {"bound": "hbm", "kernel": "kv_append_kernel", "achieved": round(gbs, 1),
                     "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 4),
                     "peak_source": f"{src} hbm_gbs", "launch_ms": round(ms, 5),
                     "algorithmic_bytes_per_launch": alg},
        "gpu_launches": steps,
    }


def subrecords(device, steps, warmup):
    """The sub-records of the default line (each measured on its own, after
    the headline, on the same GPU)."""
    records = {}
    for name, fn in (("config3", lambda: measure_config3(device, steps, warmup)),
                     ("config5_bs16", lambda: measure_config5(device, 16, steps, warmup)),
                     ("config5_bs256", lambda: measure_config5(device, 256, steps, warmup)),
                     ("prefill_long", lambda: measure_prefill_long(device, steps, warmup)),
                     ("append_64k", lambda: measure_append(device, steps, warmup))):
        records[name] = fn()
        torch.cuda.empty_cache()
    return records


def run_subrecord(args):
    """One of the default line's sub-records on its own (1 GPU), e.g. for a
    profiler capture of just that kernel."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    fn = {"config5_bs16": lambda: measure_config5(device, 16, args.steps, args.warmup),
          "config5_bs256": lambda: measure_config5(device, 256, args.steps, args.warmup),
          "prefill_long": lambda: measure_prefill_long(device, args.steps, args.warmup),
          "append_64k": lambda: measure_append(device, args.steps, args.warmup)}[args.workload]
    rec = fn()
    line = {"metric": f"{args.workload} ({rec['unit']})", "value": rec["value"],
            "unit": rec["unit"], "n_gpus": 1, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": rec["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic", "config": {"workload": rec["workload"]},
            "roofline": rec["roofline"], "gpu_launches": rec["gpu_launches"]}
    print(json.dumps(line), flush=True)


def run_config3(args):
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    rec = measure_config3(device, args.steps, args.warmup, fp8=args.kv_dtype == "fp8")
    line = {"metric": METRIC + " (config 3 mixed step)", "value": rec["value"], "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
            "ms_per_step": rec["ms_per_step"], "serial_ms_per_step": rec["serial_ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16 (KV cache fp8-e4m3)" if args.kv_dtype == "fp8" else "bf16",
            "data": "synthetic",
            "config": {"workload": rec["workload"],
                       "l2": "decode streams 2.1 GB per step between prefill launches"},
            "roofline": rec["roofline"], "roofline_prefill": rec["roofline_prefill"],
            "gpu_launches": rec["gpu_launches"]}
    print(json.dumps(line), flush=True)


def run_flashinfer_comparator(args):
    """Config 2 decode through FlashInfer's paged decode wrapper, set up the
    way the reference's FlashInferBackend sets it up (NHD, backend "auto",
    bf16 q/kv/o, CSR page indices from the block tables,
    nanovllm/layers/attention_backend.py:544-548, 726-758, 827-839), timed
    with CUDA events on the same inputs as our decode kernel, plus the
    max-abs difference between the two outputs."""
    import flashinfer

    import workloads
    from my_vllm_b200 import B200PagedBackend

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    w = workloads.config2(device=device, batch=args.batch)
    B, bs = w.num_seqs, w.block_size
    counts = torch.tensor(w.block_counts, dtype=torch.int32, device=device)
    indptr = torch.zeros(B + 1, dtype=torch.int32, device=device)
    indptr[1:] = torch.cumsum(counts, 0)
    width = w.block_tables.size(1)
    mask = torch.arange(width, device=device)[None, :] < counts[:, None]
    indices = w.block_tables[mask].contiguous()
    last = ((w.seq_lens - 1) % bs + 1).to(torch.int32)
    workspace = torch.zeros(128 << 20, dtype=torch.uint8, device=device)
    wrapper = flashinfer.BatchDecodeWithPagedKVCacheWrapper(workspace, kv_layout="NHD",
                                                            backend="auto")
    wrapper.plan(indptr, indices, last, w.num_q_heads, w.num_kv_heads, HEAD_DIM, bs,
                 pos_encoding_mode="NONE", q_data_type=torch.bfloat16,
                 kv_data_type=torch.bfloat16, o_data_type=torch.bfloat16)
    out_fi = torch.empty_like(w.q)
    stream = torch.cuda.current_stream(device)

    def fi():
        wrapper.run(w.q, (w.k_cache, w.v_cache), out=out_fi)

    backend = B200PagedBackend(w.num_q_heads, w.num_kv_heads, HEAD_DIM, bs, torch.bfloat16)
    plan = backend.build_plan(w.common_metadata())

    def ours():
        return backend.forward(w.q, w.key, w.value, w.k_cache, w.v_cache, plan)

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / args.steps

    fi_ms = timed(fi)
    our_ms = timed(ours)
    diff = float((ours().float() - out_fi.float()).abs().max())
    kv = w.kv_bytes_read()

    # config 3's prefill part through the prefill wrapper (causal, NHD)
    w3 = workloads.config3(device=device)
    nP = w3.num_prefill_seqs
    P = int(w3.extra["qsl_host"][nP])
    counts3 = torch.tensor(w3.block_counts[:nP], dtype=torch.int32, device=device)
    kv_indptr3 = torch.zeros(nP + 1, dtype=torch.int32, device=device)
    kv_indptr3[1:] = torch.cumsum(counts3, 0)
    mask3 = torch.arange(w3.block_tables.size(1), device=device)[None, :] < counts3[:, None]
    indices3 = w3.block_tables[:nP][mask3].contiguous()
    last3 = ((w3.seq_lens[:nP] - 1) % bs + 1).to(torch.int32)
    pwrap = flashinfer.BatchPrefillWithPagedKVCacheWrapper(workspace, kv_layout="NHD",
                                                           backend="auto")
    pwrap.plan(w3.query_start_loc[: nP + 1], kv_indptr3, indices3, last3, 32, 8, HEAD_DIM, bs,
               causal=True, q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16,
               o_data_type=torch.bfloat16)
    out3_fi = torch.empty_like(w3.q[:P])
    out3 = torch.empty_like(w3.q[:P])
    from my_vllm_b200 import ops

    def fi_prefill():
        pwrap.run(w3.q[:P], (w3.k_cache, w3.v_cache), out=out3_fi)

    def our_prefill():
        ops.paged_prefill(w3.q[:P], w3.k_cache, w3.v_cache, w3.block_tables[:nP],
                          w3.seq_lens[:nP], w3.query_start_loc[: nP + 1], out3, 512,
                          HEAD_DIM ** -0.5, num_seqs=nP)

    fi_pre_ms = timed(fi_prefill)
    our_pre_ms = timed(our_prefill)
    pre_diff = float((out3.float() - out3_fi.float()).abs().max())
    line = {
        "impl": "flashinfer-comparator", "metric": "paged decode HBM GB/s (decode launch only)",
        "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"config2 decode, B {B}, ctx {CONTEXT}, Hq 32 / Hkv 8, bs 16",
                   "flashinfer": flashinfer.__version__,
                   "wrapper": "BatchDecodeWithPagedKVCacheWrapper(NHD, backend=auto)"},
        "flashinfer_ms": round(fi_ms, 5), "flashinfer_gbs": round(kv / (fi_ms * 1e-3) / 1e9, 1),
        "ours_ms": round(our_ms, 5), "ours_gbs": round(kv / (our_ms * 1e-3) / 1e9, 1),
        "speedup": round(fi_ms / our_ms, 3), "max_abs_diff": diff,
        "prefill_config3": {"flashinfer_ms": round(fi_pre_ms, 5), "ours_ms": round(our_pre_ms, 5),
                            "speedup": round(fi_pre_ms / our_pre_ms, 3),
                            "max_abs_diff": pre_diff,
                            "wrapper": "BatchPrefillWithPagedKVCacheWrapper(NHD, backend=auto, "
                                       "causal)"},
    }
    print(json.dumps(line), flush=True)


def run_config4(args, rank, world, local_rank):
    """Config 4: Qwen3-32B heads sharded over ``world`` ranks (tp), all 64
    layers' KV append + paged decode per step, B 512, context U[1024, 8192].
    Each rank holds its own 64-layer cache shard in one allocation sized from
    the free HBM; below tp 4 the pool cannot hold every block and the block
    tables are sampled with replacement (stated in the line). value = KV +
    append bytes of all ranks / max rank step time; tokens/s = 512 / step."""
    import workloads
    from my_vllm_b200 import B200PagedBackend, ops

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=device)
    if 8 % world:
        raise SystemExit("--gpus must divide 8 KV heads")
    free, _ = torch.cuda.mem_get_info(device)
    layers = 64
    fp8 = args.kv_dtype == "fp8"
    w = workloads.config4_layers(device, tp=world, layers=layers,
                                 memory_budget=max(0, free - (12 << 30)),
                                 kv_dtype=torch.float8_e4m3fn if fp8 else None)
    Hq, Hkv = 64 // world, 8 // world
    backend = B200PagedBackend(Hq, Hkv, HEAD_DIM, BLOCK_SIZE, torch.bfloat16,
                               kv_cache_dtype=torch.float8_e4m3fn if fp8 else None)
    plan = backend.build_plan(w.common_metadata())
    caches = [w.layer(l) for l in range(layers)]
    if fp8:
        one = torch.ones(1, device=device)
        for kc, vc in caches:
            ops.register_kv_scales(kc, vc, one, one)
    stream = torch.cuda.current_stream(device)

    def step():
        for kc, vc in caches:
            ops.store_kvcache(w.key, w.value, kc, vc, w.slot_mapping)
            backend.forward(w.q, w.key, w.value, kc, vc, plan)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    sampler = None
    if rank == 0 and not args.no_clocks:
        sampler = ClockSampler(physical_gpu_indices(world))
        sampler.start()
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(device)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(device)
    wall0 = time.time()
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize(device)
    wall1 = time.time()
    barrier()
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps)
    backend.check_status()
    if sampler is not None:
        sampler.mark(wall0, wall1)
        sampler.stop()
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    per_rank = (w.kv_bytes_read_per_layer() + w.append_bytes_per_layer()) * layers
    total = per_rank * world
    hbm, src = peaks()
    per_gpu = per_rank / (ms * 1e-3) / 1e9
    n_parts = plan.metadata.decode_plan.num_parts
    line = {
        "metric": METRIC + " (config 4, 64 layers)", "value": round(total / (ms * 1e-3) / 1e9, 1),
        "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16 (KV cache fp8-e4m3)" if fp8 else "bf16",
        "data": "synthetic",
        "tokens_per_s": round(512 / (ms * 1e-3), 1),
        "config": {"workload": "config4: Qwen3-32B heads (64 q / 8 KV, D 128), 64 layers of KV "
                               "append + paged decode per step, B 512, ctx U[1024, 8192], bs 16"
                               + ("; KV pool FP8 E4M3" if fp8 else ""),
                   "parallelism": f"tp{world}: KV heads sharded, {Hq} q / {Hkv} KV heads per "
                                  "rank, no data-path collective",
                   "pool_blocks_per_layer": w.pool_blocks,
                   "block_tables": "sampled with replacement (pool smaller than the batch needs)"
                                   if w.with_replacement else "seeded permutation",
                   "decode_split": n_parts,
                   "l2": f"{per_rank / 1e9:.1f} GB of paged KV per rank per step"},
        "roofline": {"bound": "hbm", "kernel": "paged_decode_kernel + kv_append_kernel",
                     "achieved": round(per_gpu, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(per_gpu / hbm, 4), "peak_source": src},
        "gpu_launches": layers * (2 + (1 if n_parts > 1 else 0)) * args.steps,
    }
    if sampler is not None:
        line["clocks"] = sampler.summary()
    print(json.dumps(line), flush=True)


def run_rope_append(args):
    """The step before attention, fused: q/k RMSNorm + neox RoPE + KV append
    for one layer of Qwen3-8B (Hq 32, Hkv 8, D 128) over --rope-tokens new
    tokens. Algorithmic bytes per launch: read q, k, v and one cos|sin row per
    token, write rotated q and the k/v cache rows (weights and metadata are
    negligible). The engine's unfused chain (q_norm, k_norm, rotary_emb in
    torch eager, then the append) is timed beside it for context."""
    from my_vllm_b200 import ops

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    T, Hq, Hkv, D = args.rope_tokens, TOTAL_Q_HEADS, TOTAL_KV_HEADS, HEAD_DIM
    g = torch.Generator(device=device).manual_seed(4242)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, generator=g, device=device).to(torch.bfloat16)
    q = qkv[:, : Hq * D].view(T, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
    v = qkv[:, (Hq + Hkv) * D:].view(T, Hkv, D)
    max_pos = 40960
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float, device=device) / D))
    freqs = torch.outer(torch.arange(max_pos, dtype=torch.float, device=device), inv_freq)
    table = torch.cat((freqs.cos(), freqs.sin()), dim=-1).contiguous()
    positions = torch.randint(0, max_pos, (T,), generator=g, device=device)
    qw = (1 + 0.1 * torch.randn(D, generator=g, device=device)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(D, generator=g, device=device)).to(torch.bfloat16)
    num_blocks = max(2 * T // BLOCK_SIZE, 1)
    fp8 = args.kv_dtype == "fp8"
    k_cache = torch.zeros(num_blocks, BLOCK_SIZE, Hkv, D,
                          dtype=torch.float8_e4m3fn if fp8 else torch.bfloat16, device=device)
    v_cache = torch.zeros_like(k_cache)
    if fp8:
        ops.register_kv_scales(k_cache, v_cache, torch.ones(1, device=device),
                               torch.ones(1, device=device))
    slots = torch.randperm(num_blocks * BLOCK_SIZE, generator=g, device=device)[:T].to(torch.int32)
    q_out = torch.empty_like(q)
    stream = torch.cuda.current_stream(device)
    es = 2
    # reads: q, k, v rows + one cos|sin row; writes: rotated q + the k/v cache rows
    alg_bytes = (T * (Hq + 2 * Hkv) * D * es) + T * D * 4 + T * Hq * D * es + \
        T * 2 * Hkv * D * k_cache.element_size()

    def fused():
        ops.qk_norm_rope_append(q, k, v, positions, qw, kw, table, 1e-6, k_cache, v_cache,
                                slots, q_out)

    def unfused():
        def norm(x, w):
            xf = x.float()
            xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)
            return xf.to(x.dtype) * w

        def rope(x):
            cs = table[positions].unsqueeze(1)
            cos, sin = cs[..., : D // 2], cs[..., D // 2:]
            x1, x2 = x.float().chunk(2, dim=-1)
            return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), -1).to(x.dtype)

        qr = rope(norm(q, qw))
        kr = rope(norm(k, kw))
        ops.store_kvcache(kr, v, k_cache, v_cache, slots)  # FP8 pools quantise here
        return qr

    def timed(fn, steps):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        for a, b in ev:
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in ev) / steps

    clocks = None if args.no_clocks else ClockSampler(physical_gpu_indices(1))
    if clocks:
        clocks.start()
    t_begin = time.time()
    ms = timed(fused, args.steps)
    if clocks:
        clocks.mark(t_begin, time.time())
        clocks.stop()
    unfused_ms = timed(unfused, max(3, args.steps // 4))
    hbm, src = peaks()
    gbs = alg_bytes / (ms * 1e-3) / 1e9
    line = {
        "metric": "fused q/k-norm + RoPE + KV append HBM GB/s", "value": round(gbs, 1),
        "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16 (KV cache fp8-e4m3)" if fp8 else "bf16",
        "data": "synthetic",
        "tokens_per_s": round(T / (ms * 1e-3), 1),
        "config": {"workload": f"rope_append: {T} new tokens of Qwen3-8B (Hq 32, Hkv 8, D 128), "
                               "positions U[0, 40960), rope theta 1e6, bs 16, random slots",
                   "l2": f"{alg_bytes / 1e6:.0f} MB per launch (> 126 MB L2)"},
        "roofline": {"bound": "hbm", "kernel": "qk_norm_rope_append_kernel",
                     "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(gbs / hbm, 4), "peak_source": src,
                     "algorithmic_bytes_per_launch": alg_bytes},
        "unfused_torch_eager_ms": round(unfused_ms, 5),
        "gpu_launches": args.steps,
    }
    if clocks:
        line["clocks"] = clocks.summary()
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.comparator == "flashinfer":
        run_flashinfer_comparator(args)
        return
    if args.workload == "config3":
        run_config3(args)
        return
    if args.workload == "rope_append":
        run_rope_append(args)
        return
    if args.workload in ("config5_bs16", "config5_bs256", "prefill_long", "append_64k"):
        run_subrecord(args)
        return
    if args.workload == "config4":
        if args.gpus > 1 and "WORLD_SIZE" not in os.environ:
            raise SystemExit("--gpus N > 1 must be launched with torchrun (one process per GPU)")
        run_config4(args, rank, int(os.environ.get("WORLD_SIZE", "1")), local_rank)
        return
    if world != args.gpus and "WORLD_SIZE" not in os.environ:
        world = args.gpus
    if world > 1 and "WORLD_SIZE" not in os.environ:
        raise SystemExit("--gpus N > 1 must be launched with torchrun (one process per GPU)")
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
