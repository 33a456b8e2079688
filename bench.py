#!/usr/bin/env python
"""Benchmark of the B200 kvcache path: LMCache-style multi-layer batch copy.

Workload ("cfg2"): Llama-3-8B KV shape, bf16, 32 layers,
8 kv heads x 128, block_size 16, 32768 blocks per layer held as an LMCache layer
list of ``[2, NB, BS, NH, HS]`` tensors (64 GiB for all 32 layers); 64 requests
with lengths uniform in [256, 4096] whose block tables come from one random
permutation.  One step = gather every layer into the contiguous buffer
``[2, L, T, 1024]`` (``lmcache_kv_paged_to_buffer``) and scatter it back
(``lmcache_kv_buffer_to_paged``), all layers in one launch each.

Metric: achieved HBM GB/s of algorithmic bytes (payload read + written, index
arrays excluded) = 4 * (2 * L * T * 1024 * 2 B) per step / device time.

Multi-GPU (torchrun, one process per GPU): the 32-layer model is layer-sharded,
rank r owning layers [r*32/N, (r+1)*32/N) (strong scaling: the total work is the
same at every N); no collective runs on the data path.  The timed region is
bracketed by barriers + device syncs, the max over ranks is the step time, and
``value`` = all ranks' bytes / that time.  At N >= 2 the run also measures the
config-5 block migration (GPU 0 -> GPUs 1..N-1 over NVLink) with a byte check.

After the headline the same run times every other config of the path (cfg1,
cfg2-tile, cfg3 E4M3 / E5M2 at 8192 and 256 tokens, cfg4, cfg5, cfg5-fp8) with
fewer steps and reports them in a ``configs`` block of the same JSON line.

``--impl reference`` times the reference algorithm's CPU restatement
(``oracle/``) on the host cores instead (rank 0 only under torchrun).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "musa-aiter_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "KV gather/scatter/FP8-store HBM GB/s (% of 8 TB/s) at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
PEER_COPY_GBS = 770.0  # measured peer copy per direction on this pool's B200s (NVLink 5)
CONFIG_NAMES = ("cfg1", "cfg2-tile", "cfg3-e4m3-8192", "cfg3-e5m2-8192", "cfg3-e4m3-256", "cfg3-e5m2-256",
                "cfg4", "cfg5", "cfg5-fp8")


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("native", "reference"), default="native")
    ap.add_argument("--layers", type=int, default=32,
                    help="model layers (32 = configs[1]); torchrun ranks split them (strong scaling)")
    ap.add_argument("--blocks", type=int, default=None,
                    help="cache blocks (default 32768 for cfg2/tile/FP8 workloads, 8192 cfg4, 16384 cfg5/cfg5m)")
    ap.add_argument("--requests", type=int, default=None, help="requests (default 64 for cfg2, 128 cfg4, 256 cfg5)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the post-run byte check of the headline")
    ap.add_argument("--configs", default="all",
                    help="comma-separated configs for the 'configs' block of the default run ('all' or 'none'): "
                         + ", ".join(CONFIG_NAMES))
    ap.add_argument("--config-steps", type=int, default=5, help="timed steps per config of the 'configs' block")
    ap.add_argument("--no-migration", action="store_true", help="skip the cfg5m migration leg at N >= 2")
    ap.add_argument("--cpu-requests", type=int, default=8, help="requests in the bounded CPU sample")
    ap.add_argument("--workload", default="cfg2",
                    choices=("cfg2", "cfg1", "cfg1-tile", "cfg2-tile", "cfg3-e4m3", "cfg3-e5m2", "cfg4", "cfg5",
                             "cfg5-fp8", "cfg5m", "ops"),
                    help="cfg2 (default) is the headline run; the others time one config alone (profiling), "
                         "'ops' times each remaining kvcache op once")
    ap.add_argument("--tokens", type=int, default=8192, help="cfg3 batch tokens (256 decode / 8192 prefill)")
    ap.add_argument("--mla-layers", type=int, default=8,
                    help="layers of --workload cfg5 / cfg5-fp8 run alone (the configs block uses the 61-layer model)")
    ap.add_argument("--ops", default=None,
                    help="--workload ops: comma-separated name fragments; only the matching ops run (profiling one op)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------

BS, NH, HS = 16, 8, 128
HIDDEN = NH * HS


def request_lengths(n: int) -> list[int]:
    g = torch.Generator().manual_seed(2)
    return torch.randint(256, 4097, (n,), generator=g).tolist()


def block_slots(lens: list[int], nb: int) -> torch.Tensor:
    """Per-request block tables from one permutation of the block ids (seed 1)."""
    g = torch.Generator().manual_seed(1)
    perm = torch.randperm(nb, generator=g)
    out, used = [], 0
    for n in lens:
        k = (n + BS - 1) // BS
        bt = perm[used: used + k]
        used += k
        pos = torch.arange(n)
        out.append(bt[pos // BS] * BS + pos % BS)
    if used > nb:
        raise ValueError("not enough blocks for the requests")
    return torch.cat(out).to(torch.int64)


def payload_bytes(layers: int, tokens: int) -> int:
    return 2 * layers * tokens * HIDDEN * 2


def rank_layers(total: int, world: int, rank: int) -> range:
    """Layers rank ``rank`` owns when ``total`` layers are split over ``world`` ranks (contiguous;
    the first ``total % world`` ranks take one more)."""
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return range(lo, lo + base + (1 if rank < extra else 0))


def lmcache_layer(layer: int, nb: int, dev) -> torch.Tensor:
    """Layer ``layer`` of the cfg2 LMCache list, seeded by its global index so that every layer
    holds the same values whichever rank owns it."""
    g = torch.Generator(device=dev).manual_seed(1000 + layer)
    return torch.empty((2, nb, BS, NH, HS), dtype=torch.bfloat16, device=dev).normal_(generator=g)


# ---------------------------------------------------------------------------
# measurement helpers
# ---------------------------------------------------------------------------


def load_peak() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def load_traffic(kernel: str) -> dict | None:
    """Per-unit DRAM bytes of one kernel from the committed ncu-derived table ``profiles/traffic.json``."""
    path = ROOT / "profiles" / "traffic.json"
    try:
        return json.loads(path.read_text()).get(kernel)
    except Exception:
        return None


class ClockSampler:
    """NVML sampling of SM clock and clock-event reasons during the timed region."""

    REASONS = {
        0x1: "gpu_idle",
        0x2: "applications_clocks_setting",
        0x4: "sw_power_cap",
        0x8: "hw_slowdown",
        0x10: "sync_boost",
        0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int):
        self.samples: list[int] = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _run(self):
        nv = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
            except Exception:
                pass
            time.sleep(0.002)

    def start(self):
        if self.nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self) -> dict:
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
        names = sorted(n for bit, n in self.REASONS.items() if self.reasons & bit)
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": names,
            "samples": len(self.samples),
        }


class Dist:
    """The process group of a torchrun launch (or a single process): barrier and max / sum over ranks."""

    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=self.dev)

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()

    def reduce(self, values: list[float], op: str = "max") -> list[float]:
        if self.world == 1:
            return list(values)
        import torch.distributed as dist

        t = torch.tensor(values, dtype=torch.float64, device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
        return t.tolist()

    def gather(self, values: list[float]) -> list[list[float]]:
        """Every rank's ``values`` (same length on all ranks), in rank order."""
        if self.world == 1:
            return [list(values)]
        import torch.distributed as dist

        t = torch.tensor(values, dtype=torch.float64, device=self.dev)
        out = torch.empty((self.world, len(values)), dtype=torch.float64, device=self.dev)
        dist.all_gather_into_tensor(out, t)
        return out.tolist()

    def close(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


# ---------------------------------------------------------------------------
# CPU legs (oracle restatement of the reference algorithm) and the oracle sample of the parity check
# ---------------------------------------------------------------------------


def cpu_sample(layers, nb_total: int, n_requests: int, caches_gpu=None):
    """Compacted host copy of the first ``n_requests`` requests' blocks for the given layers.

    Returns (caches as numpy uint16 [2, nb_s, BS, NH, HS] per layer, remapped slots, tokens,
    the touched block ids).  With ``caches_gpu`` (one tensor per entry of ``layers``) the values
    are the GPU caches' own blocks; otherwise seeded random.
    """
    lens = request_lengths(64)[:n_requests]
    slots = block_slots(lens, nb_total)
    blocks = torch.unique(slots // BS)
    remap = torch.full((nb_total,), -1, dtype=torch.int64)
    remap[blocks] = torch.arange(blocks.numel())
    new_slots = (remap[slots // BS] * BS + slots % BS).numpy()
    caches = []
    rng = np.random.default_rng(0)
    for i in range(len(layers)):
        if caches_gpu is not None:
            c = caches_gpu[i].index_select(1, blocks.to(caches_gpu[i].device)).cpu()
            caches.append(c.view(torch.int16).numpy().view(np.uint16))
        else:
            caches.append(rng.integers(0, 1 << 16, size=(2, blocks.numel(), BS, NH, HS), dtype=np.uint16))
    return caches, new_slots, int(slots.numel()), blocks


def cpu_step(caches, slots, mem, threads: int):
    from oracle import kv_oracle as O

    O.lmcache_list_paged_to_buffer(caches, mem, slots, threads=threads)
    O.lmcache_list_buffer_to_paged(mem, caches, slots, 0, threads=threads)


def time_cpu(caches, slots, tokens: int, steps: int, warmup: int, threads: int):
    mem = np.empty((2, len(caches), tokens, HIDDEN), dtype=np.uint16)
    for _ in range(warmup):
        cpu_step(caches, slots, mem, threads)
    t0 = time.perf_counter()
    for _ in range(steps):
        cpu_step(caches, slots, mem, threads)
    dt = (time.perf_counter() - t0) / steps
    return 4 * payload_bytes(len(caches), tokens) / dt / 1e9, dt


def verify_cfg2(args, caches, mem, slots, layers, sample) -> dict:
    """Byte check of the headline after its timed loop, at full size.

    * device: every (kv, layer) row of the gathered buffer against the cache rows its slots name,
      read with torch indexing on the device (all T tokens of this rank's layers);
    * oracle: the first ``--cpu-requests`` requests, touched blocks compacted to the host: the
      buffer against the CPU oracle's gather, then a scatter of the bit-inverted buffer through the
      public API against the oracle's scatter of the same (partly filled last blocks keep their
      other slots), after which the original rows are scattered back.
    Returns mismatch counts (rows) for this rank.
    """
    import musa_aiter as ma
    from oracle import kv_oracle as O

    dev = mem.device
    bad_dev = torch.zeros((), dtype=torch.int64, device=dev)
    for i, c in enumerate(caches):
        for kv in range(2):
            want = c[kv].view(-1, HIDDEN).index_select(0, slots)
            bad_dev += (want.view(torch.int16) != mem[kv, i].view(torch.int16)).any(1).sum()
    s_caches, s_slots, s_tok, s_blocks = sample
    got = mem[:, :, :s_tok].cpu().view(torch.int16).numpy().view(np.uint16)
    ref = np.zeros((2, len(caches), s_tok, HIDDEN), np.uint16)
    O.lmcache_list_paged_to_buffer(s_caches, ref, s_slots)
    bad_gather = int((got != ref).any(-1).sum())
    inv = (~mem[:, :, :s_tok].contiguous().view(torch.int16)).view(torch.bfloat16)
    ma.lmcache_kv_buffer_to_paged(inv, caches, slots[:s_tok], 0, BS, NH, HS)
    after, _, _, _ = cpu_sample(layers, args.blocks, min(args.cpu_requests, args.requests), caches)
    want_caches = [c.copy() for c in s_caches]
    O.lmcache_list_buffer_to_paged(inv.cpu().view(torch.int16).numpy().view(np.uint16), want_caches, s_slots)
    bad_scatter = int(sum(int((a != w).reshape(-1, HIDDEN).any(-1).sum()) for a, w in zip(after, want_caches)))
    ma.lmcache_kv_buffer_to_paged(mem[:, :, :s_tok].contiguous(), caches, slots[:s_tok], 0, BS, NH, HS)
    torch.cuda.synchronize(dev)
    return {"device_rows_checked": 2 * len(caches) * int(slots.numel()), "device_bad_rows": int(bad_dev.item()),
            "oracle_tokens": s_tok, "oracle_gather_bad_rows": bad_gather, "oracle_scatter_bad_rows": bad_scatter}


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------


def config_block(args, tokens: int, world: int) -> dict:
    per_rank = sorted({len(rank_layers(args.layers, world, r)) for r in range(world)})
    return {
        "workload": "cfg2 LMCache-style multi-layer batch copy (gather to [2,L,T,1024] + scatter back, all layers one launch each)",
        "layers_total": args.layers,
        "layers_per_rank": per_rank[0] if len(per_rank) == 1 else per_rank,
        "num_blocks": args.blocks,
        "block_size": BS,
        "kv_heads": NH,
        "head_size": HS,
        "requests": args.requests,
        "tokens": tokens,
        "cache_layout": "LMCache layer list of [2, NB, BS, NH, HS]",
        "parallelism": f"layer-sharded x{world} (strong: rank r owns layers [r*{args.layers}/{world}, (r+1)*{args.layers}/{world}))",
        "l2": "inputs larger than L2 (buffer and caches are tens of GB), no flush needed",
    }


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    n_req = min(args.cpu_requests, args.requests)
    caches, slots, tokens, _ = cpu_sample(range(args.layers), args.blocks, n_req)
    gbs, dt = time_cpu(caches, slots, tokens, max(1, args.steps), max(0, args.warmup), threads)
    sample = (f"first {n_req} of {args.requests} requests ({tokens} tokens) x all {args.layers} layers, touched blocks "
              f"compacted; the whole host (all {threads} threads) at every N")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": config_block(args, int(block_slots(request_lengths(args.requests), args.blocks).numel()), world),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_native(args) -> None:
    import musa_aiter as ma
    from musa_aiter import _native

    d = Dist()
    world, rank, dev = d.world, d.rank, d.dev
    layers = rank_layers(args.layers, world, rank)
    lens = request_lengths(args.requests)
    slots_cpu = block_slots(lens, args.blocks)
    tokens = int(slots_cpu.numel())
    slots = slots_cpu.to(dev)
    caches = [lmcache_layer(l, args.blocks, dev) for l in layers]
    mem = torch.empty((2, len(layers), tokens, HIDDEN), dtype=torch.bfloat16, device=dev)
    P = payload_bytes(len(layers), tokens)
    P_all = payload_bytes(args.layers, tokens)

    def gather():
        ma.lmcache_kv_paged_to_buffer(caches, mem, slots, BS, NH, HS)

    def scatter():
        ma.lmcache_kv_buffer_to_paged(mem, caches, slots, 0, BS, NH, HS)

    for _ in range(args.warmup):
        gather()
        scatter()
    torch.cuda.synchronize(dev)
    d.barrier()
    torch.cuda.synchronize(dev)

    sampler = ClockSampler(d.local)
    stream = torch.cuda.current_stream(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _native.launch_count()
    sampler.start()
    start.record(stream)
    for k in range(args.steps):
        ev[k][0].record(stream)
        gather()
        ev[k][1].record(stream)
        scatter()
        ev[k][2].record(stream)
    end.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    launches = _native.launch_count() - launches0
    d.barrier()
    torch.cuda.synchronize(dev)

    gather_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    scatter_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    total_ms, launches_all = d.reduce([start.elapsed_time(end), float(launches)], "max")
    step_ms = total_ms / args.steps
    value = 4 * P_all / (step_ms * 1e-3) / 1e9
    peak, peak_kind = load_peak()
    achieved = 2 * P / (gather_ms * 1e-3) / 1e9
    traffic = None
    tr = load_traffic("rows_kernel_cfg2_gather")
    if tr and "dram_bytes_per_row" in tr:
        traffic = int(tr["dram_bytes_per_row"] * 2 * len(layers) * tokens)

    sample = None
    if not (args.no_parity and (args.no_cpu_baseline or world > 1)):
        sample = cpu_sample(layers, args.blocks, min(args.cpu_requests, args.requests), caches)
    parity = None
    if not args.no_parity:
        res = verify_cfg2(args, caches, mem, slots, layers, sample)
        keys = sorted(res)
        tot = dict(zip(keys, d.reduce([float(res[k]) for k in keys], "sum")))
        bad = tot["device_bad_rows"] + tot["oracle_gather_bad_rows"] + tot["oracle_scatter_bad_rows"]
        parity = {"status": "ok" if bad == 0 else "mismatch", **{k: int(v) for k, v in tot.items()},
                  "how": "after the timed loop, on every rank: all gathered rows against torch indexing of the caches "
                         "on the device; the first requests against the CPU oracle's gather and, for a bit-inverted "
                         "buffer, its scatter (touched blocks compacted)"}

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, d, caches, mem, slots_cpu, P, P_all)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        c_caches, c_slots, c_tokens, _ = sample
        gbs, _ = time_cpu([c.copy() for c in c_caches], c_slots, c_tokens, max(1, args.steps), max(0, args.warmup), threads)
        cpu = {
            "value": round(gbs, 3),
            "unit": "GB/s",
            "cores": threads,
            "kind": "port",
            "sample": f"first {min(args.cpu_requests, args.requests)} of {args.requests} requests ({c_tokens} tokens) x {len(layers)} layers, "
                      f"touched blocks compacted; numpy restatement of the reference loops; {args.steps} steps after "
                      f"{args.warmup} warm-up (as --impl reference)",
        }
    del caches, mem, sample
    torch.cuda.empty_cache()

    configs = run_configs(args, d)
    migration = None
    if world >= 2 and not args.no_migration:
        migration = run_migration(args, d)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(step_ms, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": config_block(args, tokens, world),
            "frac_of_8tbs": round(value / world / 8000.0, 4),
            "gather_gbs": round(2 * P / (gather_ms * 1e-3) / 1e9, 2),
            "scatter_call_gbs": round(2 * P / (scatter_ms * 1e-3) / 1e9, 2),
            "roofline": {
                "bound": "hbm",
                "kernel": "rows_kernel<16> (gather launch, rank 0)",
                "achieved": round(achieved, 2),
                "peak": peak,
                "peak_source": f"{peak_kind} hbm_gbs (burst copy)",
                "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "traffic": traffic,
                "traffic_source": "profiles/traffic.json: ncu DRAM bytes per gathered row, slope between two capture sizes",
                "algorithmic_bytes_per_launch": 2 * P,
            },
            "parity": parity,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": int(launches_all),
            "clocks": clocks,
            "configs": configs,
        }
        if migration is not None:
            line["migration"] = migration
        print(json.dumps(line), flush=True)
    d.close()


def _numa_bind(dev: torch.device) -> dict:
    """Pin this rank's host threads to the CPUs of its GPU's NUMA node (pinned host buffers are then
    first touched there).  Returns what was found; a single-node host changes nothing."""
    info = {"numa_node": None, "cpus": None}
    try:
        p = torch.cuda.get_device_properties(dev)
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        node = int(Path(f"/sys/bus/pci/devices/{bus}/numa_node").read_text().strip())
        info["numa_node"] = node
        if node >= 0:
            cpus: set[int] = set()
            for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
                a, _, b = part.partition("-")
                cpus.update(range(int(a), int(b or a) + 1))
            if cpus:
                os.sched_setaffinity(0, cpus)
                info["cpus"] = f"{min(cpus)}-{max(cpus)} ({len(cpus)})"
    except Exception as exc:  # noqa: BLE001 - informational only
        info["error"] = type(exc).__name__
    return info


def run_e2e(args, d: Dist, caches, mem, slots_cpu, P, P_all):
    """End to end through the public API with HOST buffers: each step copies the slot mapping
    host->device, gathers this rank's layers, copies the buffer to pinned host memory (the LMCache
    store), copies it back and scatters it (retrieve).  Before the loop every rank measures its own
    PCIe copy rate with both directions at once (all ranks together), which bounds the step."""
    import psutil

    import musa_aiter as ma

    dev, world = d.dev, d.world
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    avail = psutil.virtual_memory().available
    if P * local_world * 1.3 > avail:
        return {"value": None, "unit": "GB/s", "skipped": f"host RAM {avail >> 30} GiB too small for {local_world} x {P >> 30} GiB pinned buffers"}
    numa = _numa_bind(dev)
    host_mem = torch.empty(mem.shape, dtype=mem.dtype, pin_memory=True)
    host_slots = slots_cpu.pin_memory()
    dev_slots = torch.empty_like(slots_cpu, device=dev)
    stream = torch.cuda.current_stream(dev)
    nl = len(caches)
    d2h_stream = torch.cuda.Stream(dev)
    h2d_stream = torch.cuda.Stream(dev)

    # PCIe ceiling: the whole buffer D2H and, at the same time, H2D, on every rank at once.
    host_mem.copy_(mem)
    torch.cuda.synchronize(dev)
    d.barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    with torch.cuda.stream(d2h_stream):
        ev[0].record(d2h_stream)
        host_mem.copy_(mem, non_blocking=True)
        ev[1].record(d2h_stream)
    with torch.cuda.stream(h2d_stream):
        ev[2].record(h2d_stream)
        mem.copy_(host_mem, non_blocking=True)
        ev[3].record(h2d_stream)
    torch.cuda.synchronize(dev)
    d2h_gbs = P / (ev[0].elapsed_time(ev[1]) * 1e-3) / 1e9
    h2d_gbs = P / (ev[2].elapsed_time(ev[3]) * 1e-3) / 1e9
    pcie = d.gather([h2d_gbs, d2h_gbs])
    d.barrier()

    # The round trip is pipelined per (kv, layer) slice of the buffer: the device->host copy of
    # slice i (store) runs on one copy stream while the host->device copy of slice i-1 (retrieve)
    # runs on another, so both PCIe directions are busy at once; layers whose slices are back are
    # scattered in groups of 4 while the rest are still in flight.
    gathered = torch.cuda.Event()
    order = [(kv, l) for l in range(nl) for kv in range(2)]
    stored = {c: torch.cuda.Event() for c in order}
    back = {c: torch.cuda.Event() for c in order}
    group = 4

    def step():
        dev_slots.copy_(host_slots, non_blocking=True)
        ma.lmcache_kv_paged_to_buffer(caches, mem, dev_slots, BS, NH, HS)
        gathered.record(stream)
        d2h_stream.wait_event(gathered)
        with torch.cuda.stream(d2h_stream):
            for c in order:
                host_mem[c].copy_(mem[c], non_blocking=True)
                stored[c].record(d2h_stream)
        with torch.cuda.stream(h2d_stream):
            for c in order:
                h2d_stream.wait_event(stored[c])
                mem[c].copy_(host_mem[c], non_blocking=True)
                back[c].record(h2d_stream)
        for l0 in range(0, nl, group):
            l1 = min(nl, l0 + group)
            for l in range(l0, l1):
                stream.wait_event(back[(0, l)])
                stream.wait_event(back[(1, l)])
            ma.lmcache_kv_buffer_to_paged(mem[:, l0:l1], caches[l0:l1], dev_slots, 0, BS, NH, HS)

    steps = max(2, min(args.steps, 5))
    step()
    torch.cuda.synchronize(dev)
    d.barrier()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize(dev)
    ms_rank = a.elapsed_time(b) / steps
    d.barrier()
    per_rank_ms = [r[0] for r in d.gather([ms_rank])]
    ms = max(per_rank_ms)
    del host_mem
    # Ceiling: per rank, its 2P bytes (P each way) at the summed rate of its two directions
    # running at once; the slowest rank bounds the step.
    ceil_ms = max(2 * P / ((h + dd) * 1e9) * 1e3 for h, dd in pcie)
    value = 4 * P_all / (ms * 1e-3) / 1e9
    ceiling = 4 * P_all / (ceil_ms * 1e-3) / 1e9
    return {
        "value": round(value, 3),
        "unit": "GB/s",
        "h2d_bytes_per_step": int(P + slots_cpu.numel() * 8),
        "d2h_bytes_per_step": int(P),
        "steps": steps,
        "ms_per_step": round(ms, 3),
        "per_rank_ms": [round(x, 2) for x in per_rank_ms],
        "pcie_gbs_per_rank": [{"h2d": round(h, 1), "d2h": round(dd, 1)} for h, dd in pcie],
        "ceiling": {"value": round(ceiling, 3), "unit": "GB/s", "frac": round(value / ceiling, 4),
                    "how": "every rank copies its whole buffer D2H and H2D at once, all ranks together; per rank "
                           "its 2P bytes move at the sum of the two directions' rates; the slowest rank bounds the "
                           "step (device work hidden)"},
        "numa": numa,
        "path": "pinned host slots -> device; lmcache_kv_paged_to_buffer (this rank's layers); buffer D2H to pinned "
                "host and H2D back per (kv, layer) slice on two copy streams (both PCIe directions at once); "
                "lmcache_kv_buffer_to_paged per 4-layer group as its slices return",
    }


# ---------------------------------------------------------------------------
# the other configs (device GB/s and roofline; the headline carries the e2e and CPU legs)
# ---------------------------------------------------------------------------


def _fresh_block_slots(lens: list[int], nb: int, bs: int, seed: int = 1) -> list[torch.Tensor]:
    """Per-request slots whose block ids are distinct within a request, drawn afresh per request."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for n in lens:
        k = (n + bs - 1) // bs
        bt = torch.randperm(nb, generator=g)[:k]
        pos = torch.arange(n)
        out.append((bt[pos // bs] * bs + pos % bs).to(torch.int64))
    return out


def fp8_sector_ceiling(slots: torch.Tensor, layers: int, t: int, peak: float) -> dict:
    """Ceiling of the FP8 store + load pair on the block_size-innermost cache with these slots.

    An FP8 head tile [HD=128][BS=16] is 2 KiB = 64 DRAM sectors of 32 B, and every token writes one
    byte into each of its 128 rows, so a token-head touches all 64 sectors of its tile.  Per layer
    and head the DRAM bytes are at least: the bf16 rows read by the store and written by the load
    (2 x T x 256 B), plus every touched tile's sectors read and written back by the store (partial
    sector writes) and read by the load (3 x tiles x 2 KiB).  Algorithmic bytes: 3 B per element
    each way."""
    tiles = int(torch.unique(slots.cpu() // BS).numel())
    alg = 2 * t * HS * 3
    dram = 2 * t * HS * 2 + 3 * tiles * HS * BS
    return {"gbs": round(alg / dram * peak, 1), "touched_blocks_per_layer": tiles,
            "dram_bytes_per_step": int(dram * NH * layers * 2), "alg_bytes_per_step": int(alg * NH * layers * 2)}


def setup_workload(args, w: str, dev, rank: int, world: int):
    """Returns (config dict, bytes per step on this rank, step callable, kernel label)."""
    import musa_aiter as ma

    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    if w in ("cfg1", "cfg1-tile"):
        nb, bs, nh, hs = 256, 16, 8, 128
        slots = block_slots([100, 513, 1024, 2047], nb).to(dev)
        t = int(slots.numel())
        if w == "cfg1":
            k = torch.randn((nb, bs, nh, hs), device=dev, generator=g).half()
            v = torch.randn((nb, bs, nh, hs), device=dev, generator=g).half()
            mem = torch.empty((2, 1, t, nh * hs), dtype=torch.float16, device=dev)

            def step():
                ma.lmcache_kv_paged_to_buffer_two_x_nl([[k], [v]], mem, slots, bs, nh, hs)
                ma.lmcache_kv_buffer_to_paged_two_x_nl(mem, [[k], [v]], slots, 0, bs, nh, hs)
            label = "rows_kernel (two_x_nl NL=1)"
        else:
            k = torch.randn((nb, nh, hs, bs), device=dev, generator=g).half()
            v = torch.randn((nb, nh, hs, bs), device=dev, generator=g).half()
            ok = torch.empty((t, nh, hs), dtype=torch.float16, device=dev)
            ov = torch.empty_like(ok)

            def step():
                ma.kv_paged_to_linear(k, v, slots, out_k=ok, out_v=ov)
                ma.kv_linear_to_paged(ok, ov, k, v, slots)
            label = "tile_run_kernel + tile_single_kernel (kv_paged_to_linear / kv_linear_to_paged)"
        cfg = {"workload": f"{w}: fp16 [256,16,8,128] K/V, sequences 100/513/1024/2047 (T={t}), gather + scatter back",
               "tokens": t, "scaling": "replicas (one per rank)"}
        return cfg, 4 * 2 * t * nh * hs * 2, step, label
    if w == "cfg2-tile":
        lay = rank_layers(args.layers, world, rank)
        nl, nb, bs, nh, hd = len(lay), args.blocks, BS, NH, HS
        lens = request_lengths(args.requests)
        slots = block_slots(lens, nb).to(dev)
        t = int(slots.numel())
        k = torch.empty((nl, nb, nh, hd, bs), dtype=torch.bfloat16, device=dev).normal_(generator=g)
        v = torch.empty_like(k).normal_(generator=g)
        buf = torch.empty((2, nl, t, nh, hd), dtype=torch.bfloat16, device=dev)

        def step():
            ma.kv_paged_to_linear_multi_layer(k, v, slots, out_k=buf[0], out_v=buf[1])
            ma.kv_linear_to_paged_multi_layer(buf[0], buf[1], k, v, slots)
        cfg = {"workload": "cfg2-tile: [L,NB,NH,HD,BS] bf16 caches <-> [2,L,T,NH,HD] buffer, multi-layer gather + scatter",
               "layers_total": args.layers, "layers_per_rank": nl, "num_blocks": nb, "tokens": t,
               "scaling": "strong (layer-sharded)"}
        return cfg, 4 * payload_bytes(nl, t), step, "tile_run_kernel (multi-layer, all layers one launch)"
    if w.startswith("cfg3"):
        fmt = w.split("-")[1]
        lay = rank_layers(args.layers, world, rank)
        nl, nb, bs, nh, hd, t = len(lay), args.blocks, BS, NH, HS, args.tokens
        gc = torch.Generator().manual_seed(1)
        slots = torch.randperm(nb * bs, generator=gc)[:t].to(dev)
        kl = (torch.randn((nl, t, nh, hd), device=dev, generator=g) * 2.0).to(torch.bfloat16)
        vl = (torch.randn((nl, t, nh, hd), device=dev, generator=g) * 2.0).to(torch.bfloat16)
        if fmt == "e4m3":
            ks = kl.float().abs().amax(dim=(1, 3)) / 448.0
            vs = vl.float().abs().amax(dim=(1, 3)) / 448.0
        else:
            ks = kl.float().abs().amax() / 57344.0
            vs = vl.float().abs().amax() / 57344.0
        k8 = torch.zeros((nl, nb, nh, hd, bs), dtype=torch.uint8, device=dev)
        v8 = torch.zeros_like(k8)
        ok = torch.empty_like(kl)
        ov = torch.empty_like(vl)

        def step():
            ma.kv_linear_to_paged_fp8_multi_layer(kl, vl, k8, v8, slots, ks, vs, fp8_format=fmt)
            ma.kv_paged_fp8_to_linear_multi_layer(k8, v8, slots, ks, vs, out_dtype=torch.bfloat16, fp8_format=fmt,
                                                  out_k=ok, out_v=ov)
        cfg = {"workload": f"{w}: bf16 [L,T,8,128] -> FP8 {fmt} [L,NB,8,128,16] cache (random unique slots) and back",
               "layers_total": args.layers, "layers_per_rank": nl, "num_blocks": nb, "tokens": t,
               "scale": "per-layer-head amax/448" if fmt == "e4m3" else "scalar amax/57344",
               "scaling": "strong (layer-sharded)",
               "_ceiling": fp8_sector_ceiling(slots, nl, t, load_peak()[0])}
        return cfg, 2 * nl * t * nh * hd * 6, step, "tile_single_fp8_kernel + tile_run_kernel (fused quantize-scatter / gather-dequant)"
    if w == "cfg4":
        nl, nb, bs, nh, hs = 10, args.blocks or 8192, 64, 8, 128
        g2 = torch.Generator().manual_seed(2)
        nreq = args.requests or 128
        lens = torch.randint(1024, 32769, (nreq,), generator=g2).tolist()
        per_req = [s.to(dev) for s in _fresh_block_slots(lens, nb, bs)]
        caches = [[torch.empty((nb, bs, nh, hs), dtype=torch.bfloat16, device=dev).normal_(generator=g) for _ in range(nl)]
                  for _ in range(2)]
        mem_full = torch.empty((2, nl, max(lens), nh * hs), dtype=torch.bfloat16, device=dev)
        mems = [mem_full[:, :, :n] for n in lens]

        def step():
            for sl, mem in zip(per_req, mems):
                ma.lmcache_kv_paged_to_buffer_two_x_nl(caches, mem, sl, bs, nh, hs)
                ma.lmcache_kv_buffer_to_paged_two_x_nl(mem, caches, sl, 0, bs, nh, hs)
        tot = sum(lens)
        cfg = {"workload": "cfg4: SGLang MP 2 x 10 x [8192,64,8,128] bf16 (one GPU's layer shard of NL=80), per-request gather + scatter",
               "requests": len(lens), "tokens": tot, "num_blocks": nb, "layers_per_rank": nl,
               "scaling": "weak (10 layers per rank: the 80-layer model's shard at N=8)"}
        return cfg, 4 * 2 * nl * tot * nh * hs * 2, step, "rows_kernel (2 x NL planes per launch)"
    if w == "cfg5":
        lay = rank_layers(61, world, rank) if args.workload == "cfg2" else range(args.mla_layers)
        nl, nb, bs, kvd, ped = len(lay), args.blocks if args.workload != "cfg2" and args.blocks else 16384, 64, 512, 64
        g2 = torch.Generator().manual_seed(2)
        nreq = args.requests if args.workload == "cfg5" else 256
        lens = torch.randint(512, 16385, (nreq,), generator=g2).tolist()
        per_req = [s.to(dev) for s in _fresh_block_slots(lens, nb, bs)]
        kvc = torch.empty((nl, nb, bs, kvd), dtype=torch.bfloat16, device=dev).normal_(generator=g)
        pec = torch.empty((nl, nb, bs, ped), dtype=torch.bfloat16, device=dev).normal_(generator=g)

        def step():
            for sl in per_req:
                okv, ope = ma.kv_paged_to_mla_linear_multi_layer(kvc, pec, sl)
                ma.kv_mla_linear_to_paged_multi_layer(okv, ope, kvc, pec, sl)
        tot = sum(lens)
        cfg = {"workload": f"cfg5: MLA flat caches [{nl},{nb},64,512]+[{nl},{nb},64,64] bf16, per-request gather + scatter",
               "requests": nreq, "tokens": tot, "num_blocks": nb, "layers_per_rank": nl,
               "scaling": "strong (61 layers split over the ranks)" if args.workload == "cfg2" else "single GPU"}
        return cfg, 4 * nl * tot * (kvd + ped) * 2, step, "rows_kernel (MLA latent + rope rows)"
    if w == "cfg5-fp8":
        lay = rank_layers(61, world, rank) if args.workload == "cfg2" else range(args.mla_layers)
        nl, nb, bs, kvd, ped = len(lay), args.blocks if args.workload != "cfg2" and args.blocks else 16384, 64, 512, 64
        g2 = torch.Generator().manual_seed(2)
        nreq = args.requests if args.workload == "cfg5-fp8" else 256
        lens = torch.randint(512, 16385, (nreq,), generator=g2).tolist()
        per_req = [s.to(dev) for s in _fresh_block_slots(lens, nb, bs)]
        row = ma.mla_fp8_row_bytes(kvd, ped)
        cache = torch.zeros((nl, nb, bs, row), dtype=torch.uint8, device=dev)
        kv_full = torch.empty((nl, max(lens), kvd), dtype=torch.bfloat16, device=dev).normal_(generator=g)
        pe_full = torch.empty((nl, max(lens), ped), dtype=torch.bfloat16, device=dev).normal_(generator=g)
        out_kv = torch.empty_like(kv_full)
        out_pe = torch.empty_like(pe_full)

        def step():
            for sl, n in zip(per_req, lens):
                ma.kv_mla_linear_to_paged_fp8_rows(kv_full[:, :n], pe_full[:, :n], cache, sl)
                ma.kv_paged_fp8_rows_to_mla_linear(cache, sl, out_kv=out_kv[:, :n], out_k_pe=out_pe[:, :n])
        tot = sum(lens)
        cfg = {"workload": f"cfg5-fp8: MLA latent+rope bf16 [{nl},T,512]+[{nl},T,64] <-> FP8 rows [{nl},{nb},64,656] "
                           "(E4M3, per-128 group scales), per-request fused quantise-scatter + gather-dequantise",
               "requests": nreq, "tokens": tot, "num_blocks": nb, "layers_per_rank": nl,
               "scaling": "strong (61 layers split over the ranks)" if args.workload == "cfg2" else "single GPU"}
        return cfg, 2 * nl * tot * (2 * (kvd + ped) + row), step, "mla_fp8_store_kernel / mla_fp8_load_kernel"
    raise ValueError(w)


def time_steps(d: Dist, step, steps: int, warmup: int) -> tuple[float, int, dict]:
    """(max-over-ranks ms per step, launches of the library on this rank, clocks) for ``steps`` steps."""
    from musa_aiter import _native

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(d.dev)
    d.barrier()
    torch.cuda.synchronize(d.dev)
    sampler = ClockSampler(d.local)
    stream = torch.cuda.current_stream(d.dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = _native.launch_count()
    sampler.start()
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize(d.dev)
    clocks = sampler.stop()
    launches = _native.launch_count() - l0
    ms = d.reduce([a.elapsed_time(b) / steps], "max")[0]
    d.barrier()
    return ms, launches, clocks


def run_configs(args, d: Dist) -> dict:
    """The ``configs`` block: every other config of the path, timed like the headline with
    ``--config-steps`` steps after 3 warm-up steps; GB/s = all ranks' bytes / max rank time."""
    if args.configs == "none":
        return {}
    names = CONFIG_NAMES if args.configs == "all" else [c for c in args.configs.split(",") if c]
    unknown = [n for n in names if n not in CONFIG_NAMES]
    if unknown:
        raise SystemExit(f"--configs: unknown {unknown}; choose from {', '.join(CONFIG_NAMES)}")
    os.environ["MUSA_AITER_SKIP_VALIDATION"] = "1"  # as in --workload runs: no host syncs in the timed loop
    peak, _ = load_peak()
    out = {}
    saved = (args.tokens, args.requests, args.blocks)
    for name in names:
        w = name
        args.requests, args.blocks = 64, 32768
        if name.startswith("cfg3"):
            w = "-".join(name.split("-")[:2])
            args.tokens = int(name.split("-")[2])
        elif name in ("cfg4", "cfg5", "cfg5-fp8"):
            args.requests, args.blocks = None, None
        cfg, nbytes, step, label = setup_workload(args, w, d.dev, d.rank, d.world)
        ms, launches, clocks = time_steps(d, step, max(1, args.config_steps), 3)
        total = d.reduce([float(nbytes)], "sum")[0]
        gbs = total / (ms * 1e-3) / 1e9
        per_gpu = gbs / d.world
        ent = {"gbs": round(gbs, 1), "ms": round(ms, 4), "frac": round(per_gpu / peak, 4), "kernel": label,
               "bytes_per_step": int(total), "launches_per_step_rank0": round(launches / max(1, args.config_steps), 1),
               "sm_mhz": clocks.get("sm_mhz"), "clock_reasons": clocks.get("reasons")}
        ceil = cfg.pop("_ceiling", None)
        if ceil is not None:
            ent["sector_ceiling"] = {**ceil, "frac": round(per_gpu / ceil["gbs"], 4),
                                     "how": "FP8 head tile = 64 DRAM sectors; store reads + writes every touched "
                                            "sector, load reads it; bf16 rows once each way"}
        ent["config"] = cfg
        out[name] = ent
        del step
        torch.cuda.synchronize(d.dev)
        torch.cuda.empty_cache()
    args.tokens, args.requests, args.blocks = saved
    return out


def _mig_pattern(layer: int, blocks: torch.Tensor, words: int) -> torch.Tensor:
    """int32 words of the source blocks ``blocks`` of layer ``layer``: a function of (layer, block,
    word) only, so a receiver can rebuild what each block must hold."""
    j = torch.arange(words, device=blocks.device, dtype=torch.int64)
    x = ((blocks.to(torch.int64)[:, None] * words + j[None, :]) * 0x9E3779B1 + layer * 0x85EBCA77) & 0xFFFFFFFF
    return (x - ((x >> 31) << 32)).to(torch.int32)


def run_migration(args, d: Dist) -> dict:
    """cfg5m: GPU 0 holds a 1,048,576-token prefill (16384 blocks x 61 MLA layers of [64, 576] bf16);
    every layer's blocks move to its owner GPU (1..N-1), landing at the owner's own block table.
    Timed like the headline (max over ranks); then every owner checks every moved block of its
    layers against the source pattern, word for word."""
    from musa_aiter.ops.kv_migration import PagedBlockMigration, layer_owners

    rank, world, dev = d.rank, d.world, d.dev
    nl, nb, bs, width = 61, 16384, 64, 576
    words = bs * width * 2 // 4
    owners = layer_owners(nl, list(range(1, world)))
    chunk = 1024
    if rank == 0:
        caches = {}
        for l in range(nl):
            c = torch.empty((nb, bs, width), dtype=torch.bfloat16, device=dev)
            flat = c.view(nb, -1).view(torch.int32)
            for b0 in range(0, nb, chunk):
                flat[b0:b0 + chunk] = _mig_pattern(l, torch.arange(b0, min(nb, b0 + chunk), device=dev), words)
            caches[l] = c
    else:
        caches = {l: torch.zeros((nb, bs, width), dtype=torch.bfloat16, device=dev) for l in range(nl) if owners[l] == rank}
    mig = PagedBlockMigration(caches, owners)
    src_ids = torch.randperm(nb, generator=torch.Generator().manual_seed(1)).to(dev)
    dst_ids = torch.randperm(nb, generator=torch.Generator().manual_seed(100 + rank)).to(dev)
    ids = src_ids if rank == 0 else dst_ids
    ms, launches, clocks = time_steps(d, lambda: mig.run(ids), max(1, min(args.config_steps, 5)), 3)
    bad = 0
    for l, c in caches.items():
        if rank == 0:
            continue
        flat = c.view(nb, -1).view(torch.int32)
        for b0 in range(0, nb, chunk):
            got = flat.index_select(0, dst_ids[b0:b0 + chunk])
            bad += int((got != _mig_pattern(l, src_ids[b0:b0 + chunk], words)).any(1).sum())
    bad_total = d.reduce([float(bad)], "sum")[0]
    block_bytes = bs * width * 2
    total = nl * nb * block_bytes
    per_owner = {r: owners.count(r) * nb * block_bytes for r in sorted(set(owners))}
    mig.close()
    del caches
    torch.cuda.empty_cache()
    gbs = total / (ms * 1e-3) / 1e9
    return {
        "workload": f"cfg5m: prefill GPU0 holds {nb * bs} tokens x {nl} MLA layers [{nb},{bs},{width}] bf16; each layer's "
                    f"blocks move to its owner GPU (1..{world - 1}) at the owner's own block table",
        "owners": {str(r): owners.count(r) for r in sorted(set(owners))},
        "transport": "row engine stores into IPC-mapped peer caches (NVLink/NVSwitch); block tables via NCCL",
        "ms": round(ms, 3),
        "bytes_per_step": total,
        "aggregate_gbs": round(gbs, 1),
        "per_owner_gbs": {str(r): round(b / (ms * 1e-3) / 1e9, 1) for r, b in per_owner.items()},
        "peak": PEER_COPY_GBS,
        "peak_source": "measured peer copy per direction per GPU on this pool (GPU0's egress bounds the step)",
        "frac": round(gbs / PEER_COPY_GBS, 4),
        "byte_check": {"status": "ok" if bad_total == 0 else "mismatch", "bad_blocks": int(bad_total),
                       "blocks_checked": nl * nb,
                       "how": "every moved block of every layer, word for word against the source pattern"},
        "sm_mhz": clocks.get("sm_mhz"),
    }


def run_workload(args) -> None:
    """One config alone (``--workload X``), for profiling and per-config runs."""
    os.environ.setdefault("MUSA_AITER_SKIP_VALIDATION", "1")
    d = Dist()
    if args.workload == "cfg5m":
        if d.world < 2:
            raise SystemExit("cfg5m (block migration) needs --gpus 2 or more")
        res = run_migration(args, d)
        if d.rank == 0:
            print(json.dumps({"metric": METRIC, "value": res["aggregate_gbs"], "unit": "GB/s", "n_gpus": d.world,
                              "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms"],
                              "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                              "data": "synthetic", "config": {"workload": res["workload"]}, "migration": res}),
                  flush=True)
        d.close()
        return
    cfg, nbytes, step, label = setup_workload(args, args.workload, d.dev, d.rank, d.world)
    ms, launches, clocks = time_steps(d, step, args.steps, args.warmup)
    total = d.reduce([float(nbytes)], "sum")[0]
    peak, kind = load_peak()
    gbs = total / (ms * 1e-3) / 1e9
    ceil = cfg.pop("_ceiling", None)
    roofline = {"bound": "hbm", "kernel": label, "achieved": round(gbs / d.world, 2), "peak": peak,
                "peak_source": f"{kind} hbm_gbs", "unit": "GB/s", "frac": round(gbs / d.world / peak, 4), "traffic": None,
                "note": "whole-step algorithmic bytes / step time (plan kernels included)"}
    if ceil is not None:
        roofline["sector_ceiling"] = {**ceil, "frac": round(gbs / d.world / ceil["gbs"], 4)}
    if d.rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": d.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": cfg.get("scaling", "strong"),
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": cfg,
            "frac_of_8tbs": round(gbs / d.world / 8000.0, 4),
            "roofline": roofline,
            "gpu_launches": int(launches), "clocks": clocks, "validation": "off in the timed loop (MUSA_AITER_SKIP_VALIDATION=1)",
        }), flush=True)
    d.close()


def run_ops_sweep(args) -> None:
    """One timing per remaining kvcache op (the rows not carried by configs 1-5): block-table
    shapes of the Llama-3-8B cache (32 layers, 8 kv heads, head_dim 128, block_size 16), inputs on
    the device, CUDA events around `--steps` calls after `--warmup` calls.  Algorithmic bytes =
    payload read + written (index vectors excluded); host<->device ops report PCIe GB/s."""
    import musa_aiter as ma
    from musa_aiter import _native

    os.environ.setdefault("MUSA_AITER_SKIP_VALIDATION", "1")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    peak, kind = load_peak()
    L, NB, NH, HD, BS = args.layers, 4096, 8, 128, 16  # --layers (default 32) shrinks the caches for profiling
    T = 16384
    res = {}

    only = [f for f in (args.ops or "").split(",") if f]

    def timed(name, bytes_, fn, pcie=False, note=""):
        if only and not any(f in name for f in only):
            return
        for _ in range(max(1, args.warmup)):
            fn()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0 = _native.launch_count()
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        torch.cuda.synchronize(dev)
        ms = a.elapsed_time(b) / args.steps
        gbs = bytes_ / (ms * 1e-3) / 1e9
        ent = {"gb_s": round(gbs, 1), "ms": round(ms, 4), "bytes": int(bytes_),
               "launches_per_call": round((_native.launch_count() - l0) / args.steps, 2)}
        if not pcie:
            ent["frac_of_hbm"] = round(gbs / peak, 3)
        if note:
            ent["shape"] = note
        res[name] = ent
        print(f"# {name}: {ent}", file=sys.stderr, flush=True)

    # block-table slots: T tokens in T/BS whole blocks drawn from a permutation
    blocks = torch.randperm(NB, generator=torch.Generator().manual_seed(1))[: T // BS]
    slots = (blocks[:, None] * BS + torch.arange(BS)[None, :]).flatten().to(dev)
    tile = f"[{L},{NB},{NH},{HD},{BS}] tile caches, {T} block-table tokens"

    # a5/a6 merged K/V rows <-> tile caches, all layers one launch
    kc = torch.empty((L, NB, NH, HD, BS), dtype=torch.bfloat16, device=dev).normal_(generator=g)
    vc = torch.empty_like(kc).normal_(generator=g)
    merged = torch.empty((L, T, 2, NH, HD), dtype=torch.bfloat16, device=dev)
    nbytes = 2 * L * T * 2 * NH * HD * 2
    timed("kv_paged_to_merged_linear_multi_layer", nbytes,
          lambda: ma.kv_paged_to_merged_linear_multi_layer(kc, vc, slots, out=merged), note=tile)
    timed("kv_merged_linear_to_paged_multi_layer", nbytes,
          lambda: ma.kv_merged_linear_to_paged_multi_layer(merged, kc, vc, slots), note=tile)

    # a13 block copies: 1024 (src, dst) pairs, all layers, K and V
    pairs = torch.stack([torch.randperm(NB, generator=torch.Generator().manual_seed(2))[:1024],
                         torch.randperm(NB, generator=torch.Generator().manual_seed(3))[:1024]], 1).to(dev)
    dk, dv = torch.empty_like(kc), torch.empty_like(vc)
    timed("kv_copy_paged_blocks", 2 * 2 * 1024 * L * NH * HD * BS * 2,
          lambda: ma.kv_copy_paged_blocks(kc, vc, dk, dv, pairs), note=f"1024 block pairs of {tile.split(' tile')[0]}")
    del dk, dv

    # a14 Flash dense load / cache-back, one layer, 32 sequences of up to 2048 tokens whose block
    # tables split one permutation of the 4096 blocks (no block shared: every byte counted moves)
    B, S = 32, 2048
    lens = torch.randint(S // 2, S + 1, (B,), generator=torch.Generator().manual_seed(4))
    bt = torch.randperm(NB, generator=torch.Generator().manual_seed(10))[: B * (S // BS)].view(B, S // BS).to(torch.int32)
    tok = int(lens.sum())
    lens_d, bt_d = lens.to(dev), bt.to(dev)
    ok = torch.empty((B, S, NH, HD), dtype=torch.bfloat16, device=dev)
    ov = torch.empty_like(ok)
    timed("kv_load_and_reshape_flash", 2 * (tok * NH * HD * 2) + 2 * B * S * NH * HD * 2,
          lambda: ma.kv_load_and_reshape_flash(kc[0], vc[0], bt_d, lens_d, max_seq_len=S, out_k=ok, out_v=ov),
          note=f"[{NB},{NH},{HD},{BS}] caches -> [{B},{S},{NH},{HD}] x2, {tok} valid tokens (zero padding written)")
    timed("kv_reshape_and_cache_back_flash", 2 * 2 * tok * NH * HD * 2,
          lambda: ma.kv_reshape_and_cache_back_flash(ok, ov, kc[0], vc[0], bt_d, lens_d), note=f"{tok} tokens x2")

    # a11 FP8 merged store / load (per-layer-head scales) and a12 FP8 Flash dequant-load
    k8 = torch.zeros((L, NB, NH, HD, BS), dtype=torch.uint8, device=dev)
    v8 = torch.zeros_like(k8)
    ks = torch.full((L, NH), 0.01, device=dev)
    vs = torch.full((L, NH), 0.02, device=dev)
    nb8 = 2 * L * T * NH * HD * 3
    timed("kv_merged_linear_to_paged_fp8_multi_layer", nb8,
          lambda: ma.kv_merged_linear_to_paged_fp8_multi_layer(merged, k8, v8, slots, ks, vs), note=tile + ", e4m3")
    timed("kv_paged_fp8_to_merged_linear_multi_layer", nb8,
          lambda: ma.kv_paged_fp8_to_merged_linear_multi_layer(k8, v8, slots, ks, vs, out=merged), note=tile + ", e4m3 -> bf16")
    timed("kv_load_and_dequantize_fp8_flash", 2 * tok * NH * HD * 1 + 2 * B * S * NH * HD * 2,
          lambda: ma.kv_load_and_dequantize_fp8_flash(k8[0], v8[0], bt_d, lens_d, 0.01, 0.02, max_seq_len=S),
          note=f"[{NB},{NH},{HD},{BS}] uint8 -> [{B},{S},{NH},{HD}] bf16 x2")
    del k8, v8, kc, vc, merged, ok, ov

    # a18 LMCache MLA buffer <-> [NL, NB, BS, 576] (all layers one launch)
    NLm, NBm, BSm, W = 8, 4096, 64, 576
    Tm = 65536
    bm = torch.randperm(NBm, generator=torch.Generator().manual_seed(5))[: Tm // BSm]
    sm = (bm[:, None] * BSm + torch.arange(BSm)[None, :]).flatten().to(dev)
    pm = torch.empty((NLm, NBm, BSm, W), dtype=torch.bfloat16, device=dev).normal_(generator=g)
    bufm = torch.empty((NLm, Tm, W), dtype=torch.bfloat16, device=dev)
    mb = 2 * NLm * Tm * W * 2
    timed("lmcache_paged_to_kv_buffer_mla", mb, lambda: ma.lmcache_paged_to_kv_buffer_mla(pm, bufm, sm),
          note=f"[{NLm},{NBm},{BSm},{W}] -> [{NLm},{Tm},{W}]")
    timed("lmcache_kv_buffer_to_paged_mla", mb, lambda: ma.lmcache_kv_buffer_to_paged_mla(bufm, pm, sm),
          note=f"[{NLm},{Tm},{W}] -> [{NLm},{NBm},{BSm},{W}]")
    del pm, bufm

    # a19 DSV4 strided block transfer: staging [NL, T, 656] <-> padded pages, mode 1 (values then scales)
    row, vb, sb = 656, 640, 16
    NLs, NBs, BSs = 8, 2048, 64
    stride = BSs * row + 256
    pages = [torch.zeros(NBs * stride, dtype=torch.uint8, device=dev) for _ in range(NLs)]
    ptrs = [t.data_ptr() for t in pages]
    nblk = 1024
    bids = torch.randperm(NBs, generator=torch.Generator().manual_seed(6))[:nblk].to(dev)
    Ts = nblk * BSs
    staging = torch.randint(0, 256, (NLs, Ts, row), dtype=torch.uint8, device=dev, generator=g)
    sbytes = 2 * NLs * Ts * row
    timed("lmcache_kv_strided_block_transfer (staging->paged)", sbytes,
          lambda: ma.lmcache_kv_strided_block_transfer(staging, ptrs, bids, 0, NLs, 0, nblk, 0, Ts, BSs, row, stride, 1, vb, sb),
          note=f"{NLs} layers x {nblk} blocks x {BSs} rows of {row} B, mode 1")
    timed("lmcache_kv_strided_block_transfer (paged->staging)", sbytes,
          lambda: ma.lmcache_kv_strided_block_transfer(staging, ptrs, bids, 1, NLs, 0, nblk, 0, Ts, BSs, row, stride, 1, vb, sb),
          note=f"{NLs} layers x {nblk} blocks x {BSs} rows of {row} B, mode 1")
    del pages, staging

    # a20 DSV4 opaque byte rows by index (single pool and layer table)
    item = 1728
    npg = 262144
    src = torch.randint(0, 256, (npg, item), dtype=torch.uint8, device=dev, generator=g)
    dst = torch.zeros_like(src)
    nrow = 131072
    si = torch.randperm(npg, generator=torch.Generator().manual_seed(7))[:nrow].to(dev)
    di = torch.randperm(npg, generator=torch.Generator().manual_seed(8))[:nrow].to(dev)
    timed("kv_copy_paged_rows", 2 * nrow * item, lambda: ma.kv_copy_paged_rows(src, dst, si, di),
          note=f"{nrow} of [{npg},{item}] uint8 rows")
    del src, dst

    # a21 HiCache: layer-first device pool -> page-first device pool, and device <-> pinned host
    Lh, P, IB = 32, 65536, 2048
    lf_k = torch.empty((Lh, P, IB // 2), dtype=torch.bfloat16, device=dev).normal_(generator=g)
    lf_v = torch.empty_like(lf_k).normal_(generator=g)
    pf_k = torch.empty((P, Lh, IB // 2), dtype=torch.bfloat16, device=dev)
    pf_v = torch.empty_like(pf_k)
    npages = 16384
    hs = torch.randperm(P, generator=torch.Generator().manual_seed(9))[:npages].to(dev)
    hd_ = torch.randperm(P, generator=torch.Generator().manual_seed(10))[:npages].to(dev)
    hb = 2 * 2 * Lh * npages * IB
    timed("hicache_transfer_kv_all_layer_lf_pf", hb,
          lambda: ma.hicache_transfer_kv_all_layer_lf_pf(lf_k, pf_k, lf_v, pf_v, hs, hd_),
          note=f"{npages} pages x {Lh} layers x {IB} B, K and V")
    del pf_k, pf_v
    hp = 4096
    host_k = torch.empty((Lh, hp, IB // 2), dtype=torch.bfloat16, pin_memory=True)
    host_v = torch.empty_like(host_k, pin_memory=True)
    hsi = hs[:hp]
    hdi = torch.arange(hp, device=dev)
    timed("hicache_transfer_kv_all_layer (device->pinned host)", 2 * Lh * hp * IB,
          lambda: ma.hicache_transfer_kv_all_layer(lf_k, host_k, lf_v, host_v, hsi, hdi), pcie=True,
          note=f"{hp} pages x {Lh} layers x {IB} B, K and V, zero-copy kernel stores over PCIe")
    del lf_k, lf_v, host_k, host_v

    # f3 write-side producers on one layer's [NB, NH, HD, BS] caches: K/V rows written into the
    # block-table slots (copy_to_kv_cache) and RoPE applied in place at those slots
    k1 = torch.empty((NB, NH, HD, BS), dtype=torch.bfloat16, device=dev).normal_(generator=g)
    v1 = torch.empty_like(k1).normal_(generator=g)
    one = f"[{NB},{NH},{HD},{BS}] caches, one layer"
    for nt in (256, T):
        sl = slots[:nt]
        kt = torch.empty((nt, NH, HD), dtype=torch.bfloat16, device=dev).normal_(generator=g)
        vt = torch.empty_like(kt).normal_(generator=g)
        timed(f"copy_to_kv_cache ({nt} tokens)", 2 * 2 * nt * NH * HD * 2,
              lambda: ma.copy_to_kv_cache(kt, vt, k1, v1, sl), note=f"{one}, {nt} block-table tokens")
        pos = torch.randint(0, 8192, (nt,), generator=torch.Generator().manual_seed(5)).to(dev)
        ang = torch.arange(8192, dtype=torch.float32, device=dev)[:, None] * torch.rand(
            HD // 2, generator=torch.Generator().manual_seed(6)).to(dev)[None, :]
        cos, sin = ang.cos(), ang.sin()
        timed(f"apply_rope_to_key_cache ({nt} tokens)", 2 * nt * NH * HD * 2,
              lambda: ma.apply_rope_to_key_cache(k1, sl, pos, cos, sin),
              note=f"{one}, {nt} block-table tokens, fp32 [8192,{HD // 2}] cos/sin (table reads excluded)")
    del k1, v1, kt, vt

    # a15 CacheGen codec on a [T, 4096] bf16 slab
    x = (torch.empty((16384, 4096), dtype=torch.bfloat16, device=dev).normal_(generator=g) * 5.0)
    timed("kv_cachegen_encode", x.numel() * (2 + 2 + 1), lambda: ma.kv_cachegen_encode(x, num_bins=256),
          note="[16384,4096] bf16, 256 bins (min/max pass + encode pass)")
    enc, cb, _ = ma.kv_cachegen_encode(x, num_bins=256)
    timed("kv_cachegen_decode", x.numel() * (1 + 2), lambda: ma.kv_cachegen_decode(enc, cb, dtype=torch.bfloat16),
          note="[16384,4096] uint8 -> bf16")
    del x, enc

    # a22 host<->device byte-copy batch (copy engines for large entries)
    host = torch.empty(1 << 30, dtype=torch.uint8, pin_memory=True)
    devb = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    n_ent = 256
    size = (1 << 30) // n_ent
    offs = [i * size for i in range(n_ent)]
    timed("lmcache_musa_memcpy_batch_async (H2D)", n_ent * size,
          lambda: ma.lmcache_musa_memcpy_batch_async([devb] * n_ent, [host] * n_ent, [size] * n_ent,
                                                     destination_offsets=offs, source_offsets=offs), pcie=True,
          note=f"{n_ent} entries of {size >> 20} MiB")
    timed("lmcache_musa_memcpy_batch_async (D2H)", n_ent * size,
          lambda: ma.lmcache_musa_memcpy_batch_async([host] * n_ent, [devb] * n_ent, [size] * n_ent,
                                                     destination_offsets=offs, source_offsets=offs), pcie=True,
          note=f"{n_ent} entries of {size >> 20} MiB")
    print(json.dumps({"metric": METRIC, "workload": "ops: one timing per remaining kvcache op", "unit": "GB/s",
                      "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "peak": peak, "peak_source": f"{kind} hbm_gbs",
                      "data": "synthetic", "validation": "off in the timed loop (MUSA_AITER_SKIP_VALIDATION=1)",
                      "ops": res}), flush=True)


def main():
    args = parse_args()
    if args.requests is None:
        args.requests = {"cfg4": 128, "cfg5": 256, "cfg5-fp8": 256}.get(args.workload, 64)
    if args.blocks is None and (args.impl == "reference" or args.workload not in ("cfg4", "cfg5", "cfg5-fp8", "cfg5m")):
        args.blocks = 32768
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "ops":
        run_ops_sweep(args)
    elif args.workload != "cfg2":
        run_workload(args)
    else:
        run_native(args)


if __name__ == "__main__":
    main()
