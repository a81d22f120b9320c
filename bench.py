"""
Benchmark of the paged-KV hot path on B200: paged decode attention over all 16
layers of Llama-3.2-1B geometry at batch 256 (config 2: the headline workload).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

A step = one decode step of the hot path: for each of the 16 layers, the
KV-append of one new token per sequence (append_kv) then paged attention over
the full history (attend) — the reference engine's two calls; the same step
with both folded into one launch per layer (B200PagedBackend.append_attend) is
timed beside it (``fused``). Workload (seeded, synthetic — the reference uses no
dataset on this path): 256 sequences with context lengths lognormal(mu =
ln 256 - 0.32, sigma = 0.8) clipped to [1, 2048] (mean ~258, p90 ~524); 16-token
blocks scattered over a pool of 90% of HBM by a seeded permutation; K, V ~ N(0,
0.5) fp16 (variance 0.5), Q ~ N(0, 1). Sequences grow by one token per step.

Output: ONE JSON line on rank 0. ``value`` = aggregate tok/s with inputs resident
in HBM (per-step CUDA graphs replayed back to back; each step reads ~2.2 GB of
KV, far larger than L2, so no flush is needed); ``e2e`` = the same metric
through the public Python API with host buffers and per-step H2D/D2H inside
the timed region; ``roofline`` = the decode kernel's algorithmic bytes per
launch / its CUDA-event-timed average launch duration vs measured HBM peak
(other legs: config 3 prefill, config 4 swap, config 5 Llama serving);
``cpu_baseline`` = the CPU oracle (the reference algorithm restated) on this
host. Multi-GPU (torchrun): independent replicas, no data-path collective.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L, HKV, HQ, D, P = 16, 8, 32, 64, 16
N_SEQ = 256
SCALE = 1.0 / 8.0
KV_STD = math.sqrt(0.5)
METRIC = "paged decode-attn tok/s/GPU & HBM GB/s %peak; KV swap GB/s; at 1/2/4/8 GPU"
UNIT = "tok/s"
WORKLOAD = ("config2: fp16 paged decode attention + KV-append, 16 layers, batch 256, "
            "Llama-3.2-1B GQA 32q/8kv/d64, 16-token blocks, lognormal ctx mean~258 p90~524 cap 2048, "
            "pool 90% of HBM scattered by seeded permutation")


def contexts(rs: np.random.RandomState, n: int = N_SEQ) -> np.ndarray:
    """Reference's length distribution (bench/capacity.py:236,303-305)."""
    return np.clip(np.round(rs.lognormal(math.log(256) - 0.32, 0.8, size=n)), 1, 2048).astype(np.int64)


# ------------------------------------------------------------------ helpers


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# Cross-rank reductions of the replica bench (device = the rank's GPU, or the
# CPU under gloo in the tests). Replicas exchange only these scalars.

def max_over_ranks(dist, ms: float, device) -> float:
    """The job's elapsed time: the slowest rank's."""
    import torch
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return ms
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(dist, vals: list[float], device) -> list[float]:
    """Aggregate rates of independent replicas."""
    import torch
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(vals)
    t = torch.tensor(vals, device=device, dtype=torch.float64)
    dist.all_reduce(t)
    return [float(x) for x in t.tolist()]


def job_gpu_ids(dist, gpu_id: str) -> str:
    """Every rank's GPU id, comma-joined in rank order (for nvidia-smi -i)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return gpu_id
    ids = [None] * dist.get_world_size()
    dist.all_gather_object(ids, gpu_id)
    return ",".join(ids)


def replica_value(n_seq: int, ws: int, steps: int, max_ms: float) -> float:
    """Whole-job tok/s: every rank decodes n_seq tokens per step; the job's
    time is the slowest rank's."""
    return n_seq * ws * steps / (max_ms / 1e3)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons of the job's GPUs (comma-separated
    UUIDs), sampled every 20 ms while the timed region runs; start() returns
    once the first sample is in, so a short timed region is still covered."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=self.f, stderr=subprocess.DEVNULL)
            t_end = time.time() + 5.0
            while time.time() < t_end and self.proc.poll() is None:
                self.f.flush()
                if os.fstat(self.f.fileno()).st_size > 0:
                    break
                time.sleep(0.01)
        except Exception:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def decode_traffic(alg_bytes: float) -> tuple[int | None, str]:
    """DRAM bytes of one decode launch: the ncu capture's DRAM bytes per
    algorithmic byte (profiles/decode_traffic.json) times this launch's
    algorithmic bytes — only while the decode kernel's sources hash to what the
    capture ran; otherwise None (stale)."""
    import hashlib

    tfile = ROOT / "profiles" / "decode_traffic.json"
    try:
        tj = json.loads(tfile.read_text())
        h = hashlib.sha256()
        for f in tj["source_files"]:
            h.update((ROOT / f).read_bytes())
        if h.hexdigest() != tj["source_sha256"]:
            return None, "stale: the decode kernel's sources changed since the ncu capture"
        return (round(float(tj["dram_bytes_per_alg_byte"]) * alg_bytes),
                f"ncu capture ({tj['capture']}): DRAM bytes per algorithmic byte x this launch's algorithmic bytes")
    except Exception as e:  # noqa: BLE001
        return None, f"unavailable ({type(e).__name__})"


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def cpu_threads() -> int:
    try:
        import threadpoolctl
        info = threadpoolctl.threadpool_info()
        n = [i.get("num_threads", 0) for i in info if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return os.cpu_count() or 1


# ------------------------------------------------------------------ CPU oracle timing


class CpuDecodeStep:
    """The CPU oracle (the reference's append_kv + attend restated in numpy,
    float32 — CPU half-precision matmul has no BLAS path) on config 2: all 16
    layers of the 256-sequence batch, each layer with its own pool slab, one new
    token per sequence per step."""

    def __init__(self, seed: int, max_steps: int):
        from oracle import OraclePool  # CPU baseline / reference arm only

        rs = np.random.RandomState(seed)
        self.ctx = contexts(rs)
        pages = (self.ctx + max_steps + P - 1) // P
        nb = int(pages.sum())
        perm = rs.permutation(nb)
        self.tables, o = [], 0
        for pg in pages:
            self.tables.append(perm[o:o + pg].tolist())
            o += pg
        self.pool = OraclePool(L, nb, P, HKV, D, dtype=np.float32)
        base_k = (rs.standard_normal(self.pool.k[0].shape) * KV_STD).astype(np.float32)
        base_v = (rs.standard_normal(self.pool.v[0].shape) * KV_STD).astype(np.float32)
        for layer in range(L):  # every layer its own slab (same values: the timing does not depend on them)
            np.copyto(self.pool.k[layer], base_k)
            np.copyto(self.pool.v[layer], base_v)
        self.q = [rs.standard_normal((N_SEQ, HQ, D)).astype(np.float32) for _ in range(L)]
        self.kn = [(rs.standard_normal((N_SEQ, HKV, D)) * KV_STD).astype(np.float32) for _ in range(L)]
        self.vn = [(rs.standard_normal((N_SEQ, HKV, D)) * KV_STD).astype(np.float32) for _ in range(L)]

    def meta(self, s: int):
        from llm_serving_layer_b200.meta import build_meta

        return build_meta(self.tables, self.ctx + s + 1, [1] * N_SEQ, P)

    def step(self, m) -> float:
        """One 16-layer step (append_kv then attend per layer); seconds."""
        from oracle import attend_reference

        slots = m.slot_mapping.numpy()
        t0 = time.perf_counter()
        for layer in range(L):
            self.pool.append_kv(layer, self.kn[layer], self.vn[layer], slots)
            attend_reference(self.q[layer], self.pool.k[layer], self.pool.v[layer], SCALE, m)
        return time.perf_counter() - t0


def cpu_decode_rate(seed: int, budget_s: float = 10.0) -> dict:
    """Whole 16-layer steps of the CPU oracle for about ``budget_s`` (at least 2)."""
    est = 2 + int(budget_s)  # steps never exceed ~1 s each on a many-core host
    cs = CpuDecodeStep(seed, est + 64)
    times = []
    t_end = time.perf_counter() + budget_s
    s = 0
    while True:
        times.append(cs.step(cs.meta(s)))
        s += 1
        if (time.perf_counter() > t_end and len(times) >= 2) or s >= est + 64:
            break
    return {"step_s": sum(times) / len(times), "steps": len(times), "cores": cpu_threads(),
            "sum_ctx": int(cs.ctx.sum())}


def cpu_swap_rate(seed: int, budget_s: float = 5.0) -> dict:
    """Config 4's swap algorithm on CPU arrays (the reference's KVSwapSpace
    restated: per-layer gather of a sequence's blocks into (L, nb, 16, 8, 64) K
    and V buffers, and the scatter back into fresh blocks), fp16, over a sample
    of the 64 victims."""
    from oracle import OraclePool

    rs = np.random.RandomState(seed)
    nb_seq, n_vict = 64, 16
    nb_pool = 2 * nb_seq * n_vict + 256
    pool = OraclePool(L, nb_pool, P, HKV, D, dtype=np.float16)
    for layer in range(L):
        pool.k[layer].fill(1)  # touch every page
        pool.v[layer].fill(1)
    perm = rs.permutation(nb_pool)
    victims = [perm[i * nb_seq:(i + 1) * nb_seq] for i in range(n_vict)]
    fresh = [perm[(n_vict + i) * nb_seq:(n_vict + i + 1) * nb_seq] for i in range(n_vict)]
    per_dir = 2 * L * nb_seq * P * HKV * D * 2  # bytes one swap moves one way (K and V, all layers)
    t_out = t_in = 0.0
    n = 0
    t_end = time.perf_counter() + budget_s
    while n < 4 * n_vict and (n < n_vict or time.perf_counter() < t_end):
        i = n % n_vict
        t0 = time.perf_counter()
        k, v = pool.swap_out(victims[i])
        t1 = time.perf_counter()
        pool.swap_in(k, v, fresh[i])
        t_in += time.perf_counter() - t1
        t_out += t1 - t0
        n += 1
    return {"d2h_gbs": round(n * per_dir / t_out / 1e9, 2), "h2d_gbs": round(n * per_dir / t_in / 1e9, 2),
            "swaps": n, "cores": 1,
            "sample": (f"{n} swap-outs and swap-ins of 1024-token victims ({per_dir / 2**20:.0f} MiB each way), "
                       "numpy fancy-index gather/scatter over a 16-layer fp16 host pool (the reference's "
                       "KVSwapSpace on CPU tensors, restated); GB/s per direction")}


def cpu_llama_rate(seed: int, budget_s: float = 10.0, n_seqs: int = 16) -> dict:
    """Config 5's decode step on the host cores at reduced scale: Llama-3.2-1B
    geometry (hidden 2048, 16 layers, 32/8 heads of 64, SwiGLU 8192, vocab
    128256, RoPE theta 500000, RMSNorm) in float32 numpy, random weights,
    ``n_seqs`` sequences with config 2's context distribution; each step
    appends one token per sequence, attends through the oracle (the
    reference's PagedTorchBackend arithmetic restated), and takes the greedy
    argmax of the logits."""
    from oracle import OraclePool, attend_reference, rope

    from llm_serving_layer_b200.meta import build_meta

    H, FF, V = 2048, 8192, 128256
    rs = np.random.RandomState(seed)
    rng = np.random.default_rng(seed)

    def w(*shape):
        return (rng.random(shape, dtype=np.float32) - 0.5) * (2.0 / math.sqrt(shape[0]))

    emb = np.empty((V, H), dtype=np.float32)  # random rows, a 1024-row template repeated
    tmpl_rows = w(1024, H)
    for r0 in range(0, V, 1024):
        emb[r0:r0 + 1024] = tmpl_rows[:min(1024, V - r0)]
    tmpl = {"qkv": w(H, (HQ + 2 * HKV) * D), "o": w(HQ * D, H), "gu": w(H, 2 * FF), "dn": w(FF, H)}
    layers = [{k: v.copy() for k, v in tmpl.items()} for _ in range(L)]  # every layer its own weights
    ctx = contexts(rs, n_seqs)
    max_steps = 256
    pages = (ctx + max_steps + P - 1) // P
    nb = int(pages.sum())
    perm = rs.permutation(nb)
    tables, o = [], 0
    for pg in pages:
        tables.append(perm[o:o + pg].tolist())
        o += pg
    pool = OraclePool(L, nb, P, HKV, D, dtype=np.float32)
    for layer in range(L):
        pool.k[layer][:] = (rs.standard_normal(pool.k[layer].shape) * KV_STD).astype(np.float32) if layer == 0 \
            else pool.k[0]
        pool.v[layer][:] = pool.k[layer]
    inv = 1.0 / (500000.0 ** (np.arange(0, D, 2, dtype=np.float32) / D))
    ang = np.arange(2048 + max_steps, dtype=np.float32)[:, None] * inv[None, :]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    toks = rs.randint(0, V, size=n_seqs)

    def norm(x):
        return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + 1e-5)

    times = []
    t_end = time.perf_counter() + budget_s
    s = 0
    while s < max_steps and (len(times) < 2 or time.perf_counter() < t_end):
        m = build_meta(tables, ctx + s + 1, [1] * n_seqs, P)
        pos, slots = m.positions.numpy(), m.slot_mapping.numpy()
        t0 = time.perf_counter()
        x = emb[toks]
        for layer in range(L):
            wl = layers[layer]
            qkv = norm(x) @ wl["qkv"]
            q = rope(qkv[:, :HQ * D].reshape(n_seqs, HQ, D), pos, cos, sin)
            k = rope(qkv[:, HQ * D:(HQ + HKV) * D].reshape(n_seqs, HKV, D), pos, cos, sin)
            v = qkv[:, (HQ + HKV) * D:].reshape(n_seqs, HKV, D)
            pool.append_kv(layer, k, v, slots)
            a = attend_reference(q, pool.k[layer], pool.v[layer], SCALE, m)
            x = x + a.reshape(n_seqs, HQ * D) @ wl["o"]
            gu = norm(x) @ wl["gu"]
            g, u = gu[:, :FF], gu[:, FF:]
            x = x + ((g / (1.0 + np.exp(-g))) * u) @ wl["dn"]
        toks = np.argmax(norm(x) @ emb.T, axis=-1)
        times.append(time.perf_counter() - t0)
        s += 1
    step_s = sum(times) / len(times)
    return {"generated_tok_per_s": round(n_seqs / step_s, 2), "ms_per_step": round(step_s * 1e3, 1),
            "steps": len(times), "cores": cpu_threads(),
            "sample": (f"{len(times)} decode steps of {n_seqs} sequences (config 5 runs 1024 per GPU), "
                       "Llama-3.2-1B geometry in float32 numpy with random weights, attention through the "
                       "oracle's restatement of PagedTorchBackend, greedy argmax; host wall clock")}


# ------------------------------------------------------------------ reference arm


def run_reference(args) -> None:
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    steps, warmup = args.steps_ref, args.warmup
    cs = CpuDecodeStep(args.seed, steps + warmup)
    times = []
    for s in range(warmup + steps):
        dt = cs.step(cs.meta(s))
        if s >= warmup:
            times.append(dt)
    step_s = sum(times) / len(times)
    value = N_SEQ / step_s
    cores = cpu_threads()
    sample = (f"every step: all 16 layers (append_kv + attend, each layer its own pool slab) over the full "
              f"256-sequence batch, float32 numpy port of PagedTorchBackend on {cores} BLAS threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": ws, "steps": steps, "warmup": warmup, "ms_per_step": round(step_s * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config_for(ws),
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_for(ws: int) -> dict:
    """The ``config`` of both arms' lines (the same keys and values)."""
    return {"workload": WORKLOAD, "global_batch": N_SEQ * ws, "seq_len": 2048, "parallelism": f"replicas{ws}",
            "l2": "inputs larger than L2 (~2.2 GB of KV read per step)"}


# ------------------------------------------------------------------ B200 arm


def build_workload(torch, bk, rs, steps_total, device):
    """Scattered tables with room for every step, history K/V filled on device."""
    from llm_serving_layer_b200.meta import build_meta

    ctx = contexts(rs)
    pages = (ctx + steps_total + P - 1) // P
    total = int(pages.sum())
    perm = torch.from_numpy(rs.permutation(bk.num_blocks)[:total].astype(np.int64))
    tables, o = [], 0
    for p in pages:
        tables.append(perm[o:o + p].tolist())
        o += p
    idx = perm.to(device)
    g = torch.Generator(device=device).manual_seed(int(rs.randint(1 << 30)))
    for layer in range(L):
        for kv in range(2):
            vals = torch.randn((total, P, HKV, D), generator=g, device=device) * KV_STD
            bk._pool[layer, kv].index_copy_(0, idx, vals.to(bk.dtype))
            del vals
    metas = [build_meta(tables, ctx + s, [1] * N_SEQ, P, device=device) for s in range(steps_total)]
    return ctx, tables, metas


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    from llm_serving_layer_b200 import B200PagedBackend, B200SwapSpace
    from llm_serving_layer_b200.meta import build_meta

    ws, rank, local = dist_env()
    host_cores = None
    if ws > 1:
        # each replica's host work (batch assembly, launches, copies) on its own share of the cores
        try:
            cores = sorted(os.sched_getaffinity(0))
            lws = int(os.environ.get("LOCAL_WORLD_SIZE", ws))
            per = max(1, len(cores) // max(1, lws))
            mine = cores[local * per:(local + 1) * per] or cores
            os.sched_setaffinity(0, mine)
            torch.set_num_threads(len(mine))
            host_cores = len(mine)
        except (AttributeError, OSError):
            host_cores = None
        args.cpu_budget = 0  # the CPU baselines are timed on rank 0 of a one-GPU run only
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    seed = args.seed + 1000 * rank
    rs = np.random.RandomState(seed)

    free, total_mem = torch.cuda.mem_get_info(device)
    block_bytes = B200PagedBackend.estimate_pool_bytes(L, 1, P, HKV, D, torch.float16)
    pool_bytes = min(int(args.pool_frac * total_mem), free - (8 << 30))
    num_blocks = max(1024, pool_bytes // block_bytes)
    bk = B200PagedBackend(L, num_blocks, P, HKV, HQ, D, device=device, dtype=torch.float16, validate="device")

    n_graphs = min(args.steps, args.max_graphs)
    steps_total = args.warmup + n_graphs
    ctx, tables, metas = build_workload(torch, bk, rs, steps_total, device)
    g = torch.Generator(device=device).manual_seed(seed)
    qs = [torch.randn((N_SEQ, HQ, D), generator=g, device=device).half() for _ in range(L)]
    ks = [(torch.randn((N_SEQ, HKV, D), generator=g, device=device) * KV_STD).half() for _ in range(L)]
    vs = [(torch.randn((N_SEQ, HKV, D), generator=g, device=device) * KV_STD).half() for _ in range(L)]
    bk.reserve_workspace(N_SEQ, max(int(m.kv_indices.shape[0]) for m in metas))

    def step_eager(m):
        bk.plan(m)
        outs = []
        for layer in range(L):
            if args.fuse:
                outs.append(bk.append_attend(layer, ks[layer], vs[layer], qs[layer], SCALE, m))
            else:
                bk.append_kv(layer, ks[layer], vs[layer], m)
                outs.append(bk.attend(qs[layer], layer, SCALE, m))
        return outs

    # warm every cache (tensor maps, occupancy, allocator) eagerly, then capture
    for m in metas[: args.warmup]:
        step_eager(m)
    torch.cuda.synchronize()
    bk.check_status()

    graphs, ev = [], []
    pool_handle = None
    for m in metas[args.warmup:]:
        bk.invalidate_plan()
        gr = torch.cuda.CUDAGraph()
        # The step's 16 appends, then its 16 decode launches back to back, with
        # one pair of event nodes around the decodes: the roofline's mean launch
        # time is (elapsed / 16) over every timed step. Each layer's append still
        # precedes its attend (the inputs of every layer are given up front, so
        # the order of the other layers' kernels does not change the work), and no
        # event node sits between two kernels of a group, where it would add its
        # own latency to the measured launches.
        evs = [(torch.cuda.Event(enable_timing=True, external=True),
                torch.cuda.Event(enable_timing=True, external=True))]
        with torch.cuda.graph(gr, pool=pool_handle):
            bk.plan(m)
            if args.fuse:
                # append + attend per layer in one launch (B200PagedBackend.append_attend)
                evs[0][0].record()
                for layer in range(L):
                    bk.append_attend(layer, ks[layer], vs[layer], qs[layer], SCALE, m)
                evs[0][1].record()
            else:
                for layer in range(L):
                    bk.append_kv(layer, ks[layer], vs[layer], m)
                evs[0][0].record()
                for layer in range(L):
                    bk.attend(qs[layer], layer, SCALE, m)
                evs[0][1].record()
        pool_handle = gr.pool()
        graphs.append(gr)
        ev.append(evs)
    for gr in graphs[: min(len(graphs), 3)]:  # graph warm-up
        gr.replay()
    torch.cuda.synchronize()

    # ---- timed region: K steps (the captured steps replayed in order, cycling)
    gpu_id = str(local)
    try:
        uuid = torch.cuda.get_device_properties(device).uuid
        gpu_id = f"GPU-{uuid}" if not str(uuid).startswith("GPU-") else str(uuid)
    except Exception:
        pass
    gpu_id = job_gpu_ids(dist, gpu_id)
    clocks = ClockSampler(gpu_id)
    if rank == 0:
        clocks.start()
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(args.steps):
        graphs[s % n_graphs].replay()
    e1.record()
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    ms = max_over_ranks(dist, e0.elapsed_time(e1), device)
    if ws > 1:
        dist.barrier()
    bk.check_status()
    ms_per_step = ms / args.steps
    value = replica_value(N_SEQ, ws, args.steps, ms)

    # ---- roofline of the decode kernel (its launches inside the graphs)
    # every timed step replays graph s % n_graphs once: weight each graph's
    # decode group by how often it ran (events keep the last replay's times)
    dur = [ev[s % n_graphs][0][0].elapsed_time(ev[s % n_graphs][0][1]) / L for s in range(args.steps)]
    avg_launch_ms = sum(dur) / len(dur)
    alg = []
    for m in metas[args.warmup:]:
        kv = m.kv_lens.sum().item()
        pages_m = int(m.kv_indices.shape[0])
        # K+V read of every token's row, Q read + O write, one 8-byte page descriptor per page;
        # with the append fused in: the new K/V rows read and written to their slots too
        alg.append(kv * HKV * D * 2 * 2 + N_SEQ * HQ * D * 2 * 2 + pages_m * 8
                   + (N_SEQ * HKV * D * 2 * 2 * 2 if args.fuse else 0))
    alg_bytes = sum(alg) / len(alg)
    peak, peak_kind = measured_peaks()
    achieved = alg_bytes / (avg_launch_ms / 1e3) / 1e9
    traffic, traffic_note = decode_traffic(alg_bytes)

    # ---- the same steps with append + attend fused into one launch per layer
    fused = None
    if args.fused_extra and not args.fuse:
        fgraphs, fev = [], []
        for m in metas[args.warmup:]:
            bk.invalidate_plan()
            gr = torch.cuda.CUDAGraph()
            evf = (torch.cuda.Event(enable_timing=True, external=True),
                   torch.cuda.Event(enable_timing=True, external=True))
            with torch.cuda.graph(gr, pool=pool_handle):
                bk.plan(m)
                evf[0].record()
                for layer in range(L):
                    bk.append_attend(layer, ks[layer], vs[layer], qs[layer], SCALE, m)
                evf[1].record()
            fgraphs.append(gr)
            fev.append(evf)
        for gr in fgraphs[:3]:
            gr.replay()
        torch.cuda.synchronize()
        fsteps = min(args.steps, 4 * n_graphs)
        if ws > 1:
            dist.barrier()
        e0.record()
        for s in range(fsteps):
            fgraphs[s % n_graphs].replay()
        e1.record()
        torch.cuda.synchronize()
        fms = max_over_ranks(dist, e0.elapsed_time(e1), device)
        bk.check_status()
        fl = [a.elapsed_time(b) / L for a, b in fev]
        falg = alg_bytes + N_SEQ * HKV * D * 2 * 2 * 2  # plus the new K/V rows read and written to their slots
        flaunch = sum(fl) / len(fl)
        fused = {"value": round(N_SEQ * ws * fsteps / (fms / 1e3), 1), "unit": UNIT, "steps": fsteps,
                 "ms_per_step": round(fms / fsteps, 4), "avg_launch_us": round(flaunch * 1e3, 2),
                 "alg_bytes_per_launch": int(falg),
                 "frac": round(falg / (flaunch / 1e3) / 1e9 / peak, 4),
                 "path": "B200PagedBackend.append_attend: KV-append folded into the decode kernel (one launch per layer)"}
        del fgraphs

    # ---- e2e: public API, host buffers, H2D + D2H inside the timed region
    e2e = run_e2e(torch, bk, tables, ctx, args, device, ws, dist, n_graphs, "device")
    host_e2e = run_e2e(torch, bk, tables, ctx, args, device, ws, dist, n_graphs, "host")
    e2e["host_meta"] = {k: host_e2e[k] for k in ("value", "ms_per_step", "h2d_bytes_per_step", "path")}
    fused_e2e = run_e2e(torch, bk, tables, ctx, args, device, ws, dist, n_graphs, "device", fused=True)
    e2e["fused"] = {k: fused_e2e[k] for k in ("value", "ms_per_step", "path")}

    line_extra = {}
    # ---- swap (config 4), rank 0 measures its own GPU's host link
    if args.swap and rank == 0:
        line_extra["swap"] = run_swap(torch, bk, args, device, tables, ctx, qs, ks, vs)
    # ---- chunked prefill with radix sharing (config 3), rank 0
    if args.prefill and rank == 0:
        line_extra["prefill"] = run_prefill(torch, bk, args, device)
    # ---- full random-init Llama-3.2-1B continuous batching (config 5), every rank a replica
    if args.llama:
        if ws > 1:
            dist.barrier()
        # the device-fed loop (the reported figure), then the host-synchronous one (the
        # step's tokens read back before the next step is built) on the same steps: the
        # first 20 timed steps' sampled tokens of the two must be the same. The second run
        # finds cuBLAS warm for every GEMM shape of these steps, which favours the sync loop.
        ll = run_llama(torch, bk, args, device, rank, feed="device", record=20)
        ll_sync = run_llama(torch, bk, args, device, rank, feed="sync", record=20)
        ll["tokens_equal_to_sync_loop"] = ll.pop("tokens") == ll_sync.pop("tokens")
        ll["sync_readback"] = {k: ll_sync[k] for k in ("generated_tok_per_s", "ms_per_step",
                                                       "forward_device_ms_per_step")}
        ll["sync_readback"]["note"] = "run second, on the same steps, with every GEMM shape already seen"
        if ws > 1:
            g, p_ = sum_over_ranks(dist, [ll["generated_tok_per_s"], ll["processed_tok_per_s"]], device)
            ll["aggregate_generated_tok_per_s"] = round(g, 1)
            ll["aggregate_processed_tok_per_s"] = round(p_, 1)
        line_extra["llama"] = ll
    if ws > 1:
        dist.barrier()

    if rank == 0:
        cpu = cpu_decode_rate(args.seed, args.cpu_budget) if args.cpu_budget > 0 else None
        cpu_line = None
        if cpu:
            cpu_line = {"value": round(N_SEQ / cpu["step_s"], 3), "unit": UNIT, "cores": cpu["cores"],
                        "kind": "port",
                        "sample": (f"{cpu['steps']} whole 16-layer steps (append_kv + attend per layer, each layer "
                                   f"its own pool slab) over the full 256-sequence batch (sum ctx "
                                   f"{cpu['sum_ctx']}), float32 numpy restatement of PagedTorchBackend")}
        if args.cpu_budget > 0 and "swap" in line_extra:
            sw_cpu = cpu_swap_rate(args.seed, args.cpu_budget / 2)
            line_extra["swap"]["cpu_baseline"] = {
                "value": sw_cpu["d2h_gbs"], "unit": "GB/s", "h2d_gbs": sw_cpu["h2d_gbs"], "cores": sw_cpu["cores"],
                "kind": "port", "sample": sw_cpu["sample"]}
        if args.cpu_budget > 0 and "llama" in line_extra:
            ll_cpu = cpu_llama_rate(args.seed, args.cpu_budget)
            line_extra["llama"]["cpu_baseline"] = {
                "value": ll_cpu["generated_tok_per_s"], "unit": "generated tok/s", "cores": ll_cpu["cores"],
                "kind": "port", "ms_per_step": ll_cpu["ms_per_step"], "sample": ll_cpu["sample"]}
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": config_for(ws),
            "pool": {"num_blocks": int(num_blocks), "pool_gb": round(bk.pool_bytes() / 1e9, 1),
                     "distinct_steps": n_graphs},
            "host_cores_per_rank": host_cores,
            "e2e": e2e,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "peak_kind": peak_kind, "kernel": "decode_kernel", "traffic_source": traffic_note,
                         "alg_bytes_per_launch": int(alg_bytes), "avg_launch_us": round(avg_launch_ms * 1e3, 2),
                         "timing": ("CUDA events inside each timed step graph around its 16 back-to-back "
                                    "decode launches; mean launch = elapsed / 16"),
                         "fused_append": bool(args.fuse)},
            "cpu_baseline": cpu_line,
            "gpu_launches": args.steps * (1 + (1 if args.fuse else 2) * L),
            "fused": fused,
            "clocks": clock_info,
            **line_extra,
        }
        print(json.dumps(line), flush=True)
    del graphs
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


# Layers of the next e2e step issued before the host waits for this step's
# outputs (measured on one B200, 200 steps, pairs of runs: 0 -> 0.706 ms per
# step, 8 -> 0.673, 12 -> 0.648-0.686, all 16 -> 0.646-0.647). The input copy of
# the step after that is issued only once the host has waited: issued with the
# early layers it started beside this step's last output copy and runs fell
# into a slow mode (0.86-1.05 ms per step) at random.
E2E_AHEAD = 16


def run_e2e(torch, bk, tables, ctx, args, device, ws, dist, n_graphs, meta_mode="device",
            fused=False) -> dict:
    """Public-API end to end: per step, the step's BatchMeta (``meta_mode``
    "device": DeviceBlockTables.build_batch_meta, the rows' lengths plus the
    blocks of rows that crossed into a new page copied in one pinned transfer
    and every field computed on the GPU; "host": build_meta on the host and one
    copy per field), the step's q/k/v for 16 layers copied from one pinned host
    buffer, append_kv + attend per layer (the reference engine's calls; with
    ``fused``, append_attend), the attention outputs copied back to pinned host
    memory, one synchronize. The copies run on two side streams (inputs and
    outputs, so both directions of the link run at once), ordered by events:
    the inputs of step s + 1 (all layers, one copy) go into a second device
    buffer while step s computes, and the outputs (written by attend into one
    buffer, out=) leave four layers at a time as soon as those layers finished.
    The next step's meta is built and planned on the host while this step's GPU
    work runs, and its first E2E_AHEAD layers are issued before the host waits
    for this step's outputs. Every step's inputs and outputs cross the link
    inside the timed region (the first timed step also copies its own; the host
    reads every step's outputs before the next step's remaining layers are
    issued). Timed with CUDA events around the whole loop."""
    from llm_serving_layer_b200 import DeviceBlockTables
    from llm_serving_layer_b200.meta import build_meta

    steps = args.e2e_steps
    base = args.warmup  # fresh lengths continue from the graph steps' start
    rs = np.random.RandomState(args.seed + 7)
    nq, nk = N_SEQ * HQ * D, N_SEQ * HKV * D
    per = nq + 2 * nk
    # all layers' inputs in one pinned buffer (layer l: q | k | v), one copy per step
    hx = torch.from_numpy(np.concatenate([
        np.concatenate([rs.standard_normal(nq), rs.standard_normal(2 * nk) * KV_STD]) for _ in range(L)
    ]).astype(np.float16)).pin_memory()
    # all layers' outputs in one device buffer and one pinned buffer, copied back in groups of layers
    GROUP = 4
    dout = torch.empty((L, N_SEQ, HQ, D), dtype=torch.float16, device=device)
    hout = torch.empty((L, N_SEQ, HQ, D), dtype=torch.float16).pin_memory()
    # two device copies of the inputs: step s + 1's are copied in while step s runs
    dx = [torch.empty_like(hx, device=device) for _ in range(2)]
    dq = [[b[l * per:l * per + nq].view(N_SEQ, HQ, D) for l in range(L)] for b in dx]
    dk = [[b[l * per + nq:l * per + nq + nk].view(N_SEQ, HKV, D) for l in range(L)] for b in dx]
    dv = [[b[l * per + nq + nk:(l + 1) * per].view(N_SEQ, HKV, D) for l in range(L)] for b in dx]
    comp = torch.cuda.current_stream(device)
    cstream = torch.cuda.Stream(device=device)  # host -> device inputs
    ostream = torch.cuda.Stream(device=device)  # device -> host outputs (the other direction of the link)
    ev_ready = [torch.cuda.Event(), torch.cuda.Event()]  # buffer b holds its step's inputs
    ev_free = [torch.cuda.Event(), torch.cuda.Event()]   # buffer b is no longer read
    for e in ev_free:
        e.record(comp)
    ev_out = [torch.cuda.Event() for _ in range(L)]
    rows = np.arange(N_SEQ, dtype=np.int32)
    ones = np.ones(N_SEQ, dtype=np.int64)
    max_pages = max(len(t) for t in tables)
    bt = DeviceBlockTables(N_SEQ, max_pages, P, bk.num_blocks, device=device, ring=3, status=bk._status)
    meta_in = {"bytes": 0, "n": 0}

    def meta_for_step(s):
        kv = ctx + base + (s % n_graphs)
        if meta_mode == "host":
            m = build_meta(tables, kv, ones, P, device=device, pin=True)
            meta_in["bytes"] += sum(int(getattr(m, f).numel() * getattr(m, f).element_size()) for f in (
                "query_lens", "cu_query_lens", "kv_lens", "positions", "last_token_ix", "kv_indptr",
                "kv_indices", "kv_last_page_len", "batch_indices", "slot_mapping"))
        else:
            nu = bt.extend_to(rows, kv, tables)  # blocks of rows that crossed into a new page
            m = bt.build_batch_meta(rows, ones, kv)
            meta_in["bytes"] += 4 * (3 * N_SEQ + 3 * nu)
        meta_in["n"] += 1
        return m

    nxt = {}
    staged = set()  # steps whose inputs were copied in

    def h2d(step):
        b = step % 2
        cstream.wait_event(ev_free[b])
        with torch.cuda.stream(cstream):
            dx[b].copy_(hx, non_blocking=True)
            ev_ready[b].record(cstream)
        staged.add(step)

    # the previous step's outputs of group g have left dout (recorded on the output stream)
    ev_gcopy = [torch.cuda.Event() for _ in range(L // GROUP)]
    for e in ev_gcopy:
        e.record(comp)
    issued = {}  # step -> layers already issued
    stop_at = [0]  # no step at or past this one is issued ahead
    # with the host assembler the per-field copies of the next meta queue behind
    # the layers issued ahead (measured slower: 275 k -> 234 k tok/s): none there
    ahead = E2E_AHEAD if meta_mode == "device" else 0

    def issue_layers(s, m, lo, hi):
        b = s % 2
        if lo == 0 and hi > 0:
            comp.wait_event(ev_ready[b])
        for layer in range(lo, hi):
            if layer % GROUP == 0:
                comp.wait_event(ev_gcopy[layer // GROUP])
            if fused:
                bk.append_attend(layer, dk[b][layer], dv[b][layer], dq[b][layer], SCALE, m, out=dout[layer])
            else:
                bk.append_kv(layer, dk[b][layer], dv[b][layer], m)
                bk.attend(dq[b][layer], layer, SCALE, m, out=dout[layer])
            if layer % GROUP == GROUP - 1:
                ev_out[layer].record(comp)
        issued[s] = hi

    last = [None]  # (step, BatchMeta) of the latest step

    def one(s):
        # step s runs with the meta built during step s - 1; the next step's meta
        # is built on the host while this step's GPU work runs (one build per step)
        m = nxt.pop(s) if s in nxt else meta_for_step(s)
        last[0] = (s, m)
        if s not in staged:
            h2d(s)
        staged.discard(s)
        b = s % 2
        lo = issued.pop(s, 0)
        issue_layers(s, m, lo, min(lo + 1, L))
        # the next step's inputs travel while this step computes; issued after
        # the first layer this call issues (so that its launches are not
        # delayed) and after the wait for the previous step's outputs (so that
        # the copy does not start beside that step's last output copy)
        h2d(s + 1)
        issue_layers(s, m, min(lo + 1, L), L)
        ev_free[b].record(comp)
        # each group of layers' outputs leaves as soon as the group is done (the
        # output stream waits for its event); issued together to switch streams once
        with torch.cuda.stream(ostream):
            for g0 in range(0, L, GROUP):
                ostream.wait_event(ev_out[g0 + GROUP - 1])
                hout[g0:g0 + GROUP].copy_(dout[g0:g0 + GROUP], non_blocking=True)
                ev_gcopy[g0 // GROUP].record(ostream)
        nxt[s + 1] = meta_for_step(s + 1)
        # plan the next step now (B200PagedBackend.plan): its host work and plan
        # kernel run while this step's GPU work drains, not before its first layer
        bk.plan(nxt[s + 1])
        if ahead and s + 1 < stop_at[0]:
            # the next step's first E2E_AHEAD layers queue behind this step on the
            # GPU while the host waits for this step's outputs: the GPU does not
            # idle through the last output copy and the host's wake-up (each of
            # those layers waits for its output group's previous copy)
            issue_layers(s + 1, nxt[s + 1], 0, ahead)
        ostream.synchronize()

    if meta_mode == "device":  # admission: each row gets the blocks of its history
        for r in range(N_SEQ):
            bt.bind(r, tables[r][:(int(ctx[r]) + base + P - 1) // P])
    stop_at[0] = 3
    for s in range(3):
        one(s)
    nxt.clear()
    staged.clear()
    issued.clear()
    stop_at[0] = steps
    torch.cuda.synchronize()
    nxt[0] = meta_for_step(0)
    meta_in.update(bytes=0, n=0)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(steps):
        one(s)
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(dist, e0.elapsed_time(e1), device)
    bk.check_status()
    # the outputs that reached the host are the attention of their step: the last
    # step's last layer, recomputed through the same call, must equal them bit for bit
    s_last, m_last = last[0]
    b = s_last % 2
    # (append_kv / append_attend already wrote the step's rows: attend alone recomputes it)
    ref = bk.attend(dq[b][L - 1], L - 1, SCALE, m_last)
    torch.cuda.synchronize()
    outputs_ok = bool(torch.equal(ref.cpu(), hout[L - 1]))
    h2d_bytes = hx.numel() * 2 + meta_in["bytes"] // max(meta_in["n"], 1)
    d2h = hout.numel() * 2
    path = (("B200PagedBackend.append_attend per layer" if fused else "B200PagedBackend.append_kv/attend per layer")
            + ", validate='device', "
            + ("DeviceBlockTables.build_batch_meta (BatchMeta fields computed on the GPU from device block "
               "tables; only new blocks travel)" if meta_mode == "device" else
               "host build_meta (one copy per BatchMeta field)")
            + " built per step (the next step's while this one runs), inputs one copy per step (one step "
              "ahead, double-buffered), outputs into one buffer (attend out=) copied back 4 layers at a time, "
              "on two side streams"
            + (f"; the next step's first {E2E_AHEAD} layers issued before waiting for this step's outputs"
               if meta_mode == "device" else ""))
    return {"value": round(N_SEQ * ws * steps / (ms / 1e3), 1), "unit": UNIT, "h2d_bytes_per_step": int(h2d_bytes),
            "d2h_bytes_per_step": int(d2h), "steps": steps, "ms_per_step": round(ms / steps, 4),
            "outputs_equal_recomputed_last_layer": outputs_ok, "path": path}


def prefill_workload(seed: int):
    """Config 3: 512 prompts, lengths U[128, 1024], in 32 families sharing a
    prefix of U[64, 512] tokens. Each family's first prompt (its owner) is
    prefilled in full; every later member references the owner's whole prefix
    blocks and copies the partial last prefix block on its first write
    (copy-on-write), then prefills from the end of the prefix. Prompts are cut
    into steps of at most 512 prompt tokens across the batch, each prompt
    contributing one contiguous range per step (the reference scheduler's
    max_prefill_tokens = 512). Returns per-step (prompt ids, starts, ends),
    the block tables, the copy-on-write pairs per step and summary counts."""
    rs = np.random.RandomState(seed)
    n_fam, per_fam, budget = 32, 16, 512
    pf = rs.randint(64, 513, size=n_fam)
    lens, fam = [], []
    for f in range(n_fam):
        for _ in range(per_fam):
            lens.append(int(rs.randint(max(128, int(pf[f]) + 1), 1025)))
            fam.append(f)
    owners = [f * per_fam for f in range(n_fam)]
    members = [i for i in range(n_fam * per_fam) if i % per_fam]
    order = owners + [members[j] for j in rs.permutation(len(members))]
    free = list(rs.permutation(1 << 20))  # block ids drawn from a scattered free list (trimmed to the pool later)
    nxt = 0
    tables, start, cow = {}, {}, {}
    for i in order:
        f, L_i = fam[i], lens[i]
        nb = (L_i + P - 1) // P
        if i in owners:
            tables[i] = free[nxt:nxt + nb]
            nxt += nb
            start[i] = 0
        else:
            own = tables[owners[f]]
            whole = int(pf[f]) // P
            t = list(own[:whole])
            if pf[f] % P:
                new = free[nxt]
                nxt += 1
                cow[i] = (own[whole], new)
                t.append(new)
            rest = nb - len(t)
            t += free[nxt:nxt + rest]
            nxt += rest
            tables[i] = t
            start[i] = int(pf[f])
    steps, cows, pos = [], [], {i: start[i] for i in order}
    queue = list(order)
    while queue:
        left, ids, st, en, cw = budget, [], [], [], []
        k = 0
        while left > 0 and k < len(queue):
            i = queue[k]
            take = min(left, lens[i] - pos[i])
            if pos[i] == start[i] and i in cow:
                cw.append(cow[i])
            ids.append(i)
            st.append(pos[i])
            en.append(pos[i] + take)
            pos[i] += take
            left -= take
            k += 1
        queue = [i for i in queue if pos[i] < lens[i]]
        steps.append((ids, st, en))
        cows.append(cw)
    total_blocks = sum((l + P - 1) // P for l in lens)
    shared = sum(int(pf[fam[i]]) // P for i in members)
    return {"steps": steps, "tables": tables, "cows": cows, "blocks_used": nxt,
            "prompt_tokens": sum(lens), "computed_tokens": sum(lens[i] - start[i] for i in order),
            "block_reuse": shared / total_blocks, "n_cow": len(cow)}


def prefill_step_work(ids, st, en) -> tuple[float, float]:
    """Algorithmic FLOPs and bytes of one prefill attention launch: FLOPs =
    4 * Hq * D * unmasked (query, key) pairs, pairs = q*s + q(q+1)/2 per
    sequence; bytes = K+V of every key read once + Q read + O written."""
    fl = by = 0.0
    for s0, e in zip(st, en):
        q = e - s0
        fl += 4 * HQ * D * (q * s0 + q * (q + 1) / 2)
        by += e * HKV * D * 2 * 2 + q * HQ * D * 2 * 2
    return fl, by


def cpu_prefill_time(work: dict, budget_s: float) -> dict:
    """CPU oracle (reference prefill attend restated in numpy, float32) on the
    first steps of the config-3 schedule, one layer each, for ~budget_s."""
    from oracle import attend_reference  # CPU baseline leg only
    from llm_serving_layer_b200.meta import build_meta

    rs = np.random.RandomState(7)
    t_end = time.perf_counter() + budget_s
    toks = secs = 0.0
    n = 0
    for ids, st, en in work["steps"]:
        tabs = [list(range(0, (e + P - 1) // P)) for e in en]  # contiguous renumbering: same arithmetic
        nb = max(len(t) for t in tabs)
        k = (rs.standard_normal((nb, P, HKV, D)) * KV_STD).astype(np.float32)
        v = (rs.standard_normal((nb, P, HKV, D)) * KV_STD).astype(np.float32)
        q = rs.standard_normal((sum(e - s for s, e in zip(st, en)), HQ, D)).astype(np.float32)
        m = build_meta(tabs, en, [e - s for s, e in zip(st, en)], P)
        t0 = time.perf_counter()
        attend_reference(q, k, v, SCALE, m)
        secs += time.perf_counter() - t0
        toks += q.shape[0]
        n += 1
        if time.perf_counter() > t_end:
            break
    return {"tok_per_s": toks / (secs * L), "steps": n, "cores": cpu_threads()}


def batched_prefill_case(args, device, perm):
    """The large-batch prefill launch: the first 512-token chunk of 64 prompts
    (cached prefix ~ U[64, 512] tokens) in one launch, their pages taken in
    order from `perm`. Returns (BatchMeta, [(prefix, chunk)], kv lengths, page
    tables)."""
    from llm_serving_layer_b200.meta import build_meta

    rs = np.random.RandomState(args.seed + 8)
    specs = [(int(rs.randint(64, 513)), 512) for _ in range(64)]
    tabs, o = [], 0
    for s0, q in specs:
        nbk = (s0 + q + P - 1) // P
        tabs.append([int(x) for x in perm[o:o + nbk]])
        o += nbk
    en = [s0 + q for s0, q in specs]
    return build_meta(tabs, en, [q for _, q in specs], P, device=device), specs, en, tabs


def run_prefill(torch, bk, args, device) -> dict:
    """Config 3 on the B200 path: every step = copy-on-write copies of the step's
    new members, then for each of the 16 layers append_kv + attend (prefill
    kernel), one CUDA graph per step, all steps replayed in order after one
    warm-up pass. Reports prompt tok/s, the attention kernel's achieved
    TFLOP/s against the measured bf16 tensor peak, and a large-batch variant
    (the first 512-token chunk of 64 prompts in one launch)."""
    from llm_serving_layer_b200.meta import build_meta

    try:
        peak = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
        peak_kind = "measured"
    except Exception:
        peak, peak_kind = 1590.0, "fallback"
    work = prefill_workload(args.seed + 3)
    perm = np.random.RandomState(args.seed + 5).permutation(bk.num_blocks)
    g = torch.Generator(device=device).manual_seed(args.seed + 6)
    # large-batch variant (run first, so its launches are the first prefill launches of the
    # process): the first 512-token chunk of 64 prompts (cached prefix s ~ U[64, 512]) in one launch
    m, specs, en, _ = batched_prefill_case(args, device, perm)
    qbig = torch.randn((sum(q for _, q in specs), HQ, D), generator=g, device=device).half()
    bk.invalidate_plan()
    bk.plan(m)
    for _ in range(3):
        bk.attend(qbig, 0, SCALE, m)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    reps = 10
    for r in range(reps):
        bk.attend(qbig, r % L, SCALE, m)
    e1.record()
    torch.cuda.synchronize()
    bk.check_status()
    us = e0.elapsed_time(e1) * 1e3 / reps
    fl, _ = prefill_step_work(None, [s for s, _ in specs], en)
    batched = {"us_per_launch": round(us, 1), "tflops": round(fl / us / 1e6, 1), "frac": round(fl / us / 1e6 / peak, 4),
               "kernel": "prefill_tc_lean_kernel (tcgen05; three persistent CTAs per SM)"}
    del qbig
    if work["blocks_used"] > bk.num_blocks:
        return {"skipped": f"pool has {bk.num_blocks} blocks, config 3 needs {work['blocks_used']}",
                "batched_64x512": batched}
    remap = {}
    def blk(b):
        if b not in remap:
            remap[b] = int(perm[len(remap)])
        return remap[b]
    tables = {i: [blk(b) for b in t] for i, t in work["tables"].items()}
    cows = [[(blk(a), blk(b)) for a, b in cw] for cw in work["cows"]]
    TMAX = 512
    qb = [torch.randn((TMAX, HQ, D), generator=g, device=device).half() for _ in range(L)]
    kb = [(torch.randn((TMAX, HKV, D), generator=g, device=device) * KV_STD).half() for _ in range(L)]
    vb = [(torch.randn((TMAX, HKV, D), generator=g, device=device) * KV_STD).half() for _ in range(L)]
    metas, works = [], []
    for ids, st, en in work["steps"]:
        tabs = [tables[i][:(e + P - 1) // P] for i, e in zip(ids, en)]
        metas.append(build_meta(tabs, en, [e - s for s, e in zip(st, en)], P, device=device))
        works.append(prefill_step_work(ids, st, en))
    graphs, evs = [], []
    pool_handle = None
    for m, cw in zip(metas, cows):
        T = int(m.positions.shape[0])
        for a, b in cw:  # eager first pass: warms caches, checks the kernel path
            bk.copy_block(a, b)
        bk.invalidate_plan()
        bk.plan(m)
        for layer in range(L):
            bk.append_kv(layer, kb[layer][:T], vb[layer][:T], m)
            bk.attend(qb[layer][:T], layer, SCALE, m)
        assert bk.last_kernel == "prefill", bk.last_kernel
    torch.cuda.synchronize()
    bk.check_status()
    for m, cw in zip(metas, cows):
        T = int(m.positions.shape[0])
        bk.invalidate_plan()
        gr = torch.cuda.CUDAGraph()
        # copies, plan and the 16 appends, then the 16 attends back to back inside
        # one event pair (mean attend launch = elapsed / 16), as in the decode leg
        ev = [(torch.cuda.Event(enable_timing=True, external=True),
               torch.cuda.Event(enable_timing=True, external=True))]
        with torch.cuda.graph(gr, pool=pool_handle):
            for a, b in cw:
                bk.copy_block(a, b)
            bk.plan(m)
            for layer in range(L):
                bk.append_kv(layer, kb[layer][:T], vb[layer][:T], m)
            ev[0][0].record()
            for layer in range(L):
                bk.attend(qb[layer][:T], layer, SCALE, m)
            ev[0][1].record()
        pool_handle = gr.pool()
        graphs.append(gr)
        evs.append(ev)
    for gr in graphs:
        gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for gr in graphs:
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    bk.check_status()
    ms = e0.elapsed_time(e1)
    attn_ms = sum(a.elapsed_time(b) for ev in evs for a, b in ev)
    flops = sum(w[0] for w in works) * L
    achieved = flops / (attn_ms / 1e3) / 1e12
    out = {
        "workload": ("config3: 512 prompts U[128,1024] in 32 families sharing a U[64,512]-token prefix "
                     "(whole blocks shared through the tables, partial block copy_block'd on first write), "
                     "steps of <= 512 prompt tokens, 16 layers append_kv + causal prefill attention, fp16"),
        "steps": len(graphs), "computed_prompt_tokens": work["computed_tokens"],
        "prompt_tokens": work["prompt_tokens"], "block_reuse": round(work["block_reuse"], 3),
        "copy_on_write": work["n_cow"],
        "tok_per_s": round(work["computed_tokens"] / (ms / 1e3), 1),
        "prompt_tok_per_s_incl_cached": round(work["prompt_tokens"] / (ms / 1e3), 1),
        "ms_total": round(ms, 3), "attn_ms_total": round(attn_ms, 3),
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "kernel": "prefill_tc_kernel (tcgen05; one CTA per tile, key blocks split over two groups of the "
                               "CTA in launches of at most one CTA per SM)",
                     "avg_launch_us": round(attn_ms * 1e3 / (len(graphs) * L), 2),
                     "timing": "CUDA events around each step's 16 back-to-back attend launches"},
        "batched_64x512": batched,
    }
    del graphs
    if args.cpu_budget > 0:
        c = cpu_prefill_time(work, min(args.cpu_budget, 10.0))
        out["cpu_baseline"] = {"value": round(c["tok_per_s"], 2), "unit": "tok/s", "cores": c["cores"],
                               "kind": "port",
                               "sample": (f"first {c['steps']} steps of the schedule, one layer each, float32 "
                                          "numpy restatement of PagedTorchBackend.attend (prefill branch); "
                                          "tok/s scaled to 16 layers, attention only")}
    return out


def run_swap(torch, bk, args, device, tables, ctx, qs, ks, vs) -> dict:
    """Config 4: 64 victims x 1024 tokens (64 blocks each, scattered over blocks
    the decode workload does not use), swap-out to pinned host and swap-in to
    fresh blocks, bit-exact spot check; first alone, then overlapped with a
    batch-128 decode step (16 layers, append + attend, one CUDA graph) replayed
    back to back on the compute stream for as long as the transfers run."""
    from llm_serving_layer_b200 import B200SwapSpace
    from llm_serving_layer_b200.meta import build_meta

    class Blocks:  # the block-manager view the swap space reads
        def __init__(self, ids, n):
            self.block_ids, self.num_tokens, self.seq_id, self.is_freed = list(ids), n, 0, False

    rs = np.random.RandomState(args.seed + 4)
    victims, toks = 64, 1024
    nbv = toks // P
    used = set(b for t in tables for b in t)
    free = [b for b in rs.permutation(bk.num_blocks).tolist() if b not in used][: 2 * victims * nbv]
    src = [free[i * nbv:(i + 1) * nbv] for i in range(victims)]
    dst = [free[(victims + i) * nbv:(victims + i + 1) * nbv] for i in range(victims)]
    sw = B200SwapSpace(bk, staging_bytes=256 << 20, synchronous=False)
    per_dir = victims * sw.bytes_for(nbv)

    # host-link peak: one contiguous 1 GiB pinned <-> device copy per direction
    # (cudaMemcpyAsync on a side stream, CUDA events, best of 5)
    link = {}
    hbuf = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dbuf = torch.empty(1 << 30, dtype=torch.uint8, device=device)
    ls = torch.cuda.Stream(device=device)
    for name, dst_t, src_t in (("d2h", hbuf, dbuf), ("h2d", dbuf, hbuf)):
        best = None
        for _ in range(6):
            a_, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(ls):
                a_.record(ls)
                dst_t.copy_(src_t, non_blocking=True)
                b_.record(ls)
            ls.synchronize()
            t = a_.elapsed_time(b_)
            best = t if best is None else min(best, t)
        link[name] = round((1 << 30) / (best / 1e3) / 1e9, 2)
    del hbuf, dbuf

    # the concurrent decode: first 128 sequences of the config-2 batch, one step
    nd = 128
    m = build_meta([t for t in tables[:nd]], ctx[:nd], [1] * nd, P, device=device)
    bk.invalidate_plan()
    bk.plan(m)
    for layer in range(L):
        bk.append_kv(layer, ks[layer][:nd], vs[layer][:nd], m)
        bk.attend(qs[layer][:nd], layer, SCALE, m)
    gr = torch.cuda.CUDAGraph()
    bk.invalidate_plan()
    with torch.cuda.graph(gr):
        bk.plan(m)
        for layer in range(L):
            bk.append_kv(layer, ks[layer][:nd], vs[layer][:nd], m)
            bk.attend(qs[layer][:nd], layer, SCALE, m)
    for _ in range(3):
        gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 200
    e0.record()
    for _ in range(reps):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    alone_ms = e0.elapsed_time(e1) / reps

    def once(with_decode, sw=sw):
        torch.cuda.synchronize()
        steps = {"out": 0, "in": 0}

        def drive(kind, issue, handles_or_none):
            n = 0
            t0 = time.perf_counter()
            e0.record()
            for i in range(victims):
                issue(i)
                if with_decode:
                    gr.replay()
                    n += 1
            if with_decode:
                while not all(sw._lib.pkv_swapper_done(sw._sw, t) for t in handles_or_none()):
                    for _ in range(4):  # keep the compute stream busy, the host at most 4 steps ahead
                        gr.replay()
                        n += 1
                    torch.cuda.current_stream().synchronize()
            e1.record()
            sw.wait()
            torch.cuda.synchronize()
            steps[kind] = n
            return time.perf_counter() - t0, (e0.elapsed_time(e1) / n if n else None)

        hs = []
        t_out, dec_out = drive("out", lambda i: hs.append(sw.swap_out(f"v{i}", Blocks(src[i], toks))),
                               lambda: [h.ticket for h in hs if h.ticket])
        tick = []

        def issue_in(i):
            sw.swap_in(hs[i], Blocks(dst[i], toks))
            tick.append(sw._pending[-1][0] if sw._pending else 0)
        t_in, dec_in = drive("in", issue_in, lambda: [t for t in tick if t])
        return hs, t_out, t_in, dec_out, dec_in, steps

    hs, _, _, _, _, _ = once(False)
    for h in hs:
        sw.release(h)
    hs, t_out, t_in, _, _, _ = once(False)
    ok = True
    for i in range(0, victims, 9):  # bit-exact spot check of every 9th victim, all layers
        ok = ok and bool(torch.equal(bk._pool[:, :, src[i]], bk._pool[:, :, dst[i]]))
    for h in hs:
        sw.release(h)
    hs, to2, ti2, dec_out, dec_in, steps = once(True)
    for i in range(0, victims, 9):
        ok = ok and bool(torch.equal(bk._pool[:, :, src[i]], bk._pool[:, :, dst[i]]))
    for h in hs:
        sw.release(h)
    # the same with staging that holds the whole swap: no gather waits for an
    # earlier victim's host copy, so the compute stream waits only for gathers
    big = B200SwapSpace(bk, staging_bytes=int(per_dir), synchronous=False)
    hs, to3, ti3, dec_out3, dec_in3, steps3 = once(True, big)
    for i in range(0, victims, 9):
        ok = ok and bool(torch.equal(bk._pool[:, :, src[i]], bk._pool[:, :, dst[i]]))
    for h in hs:
        big.release(h)
    del big
    bk.check_status()
    del gr
    return {"victims": victims, "tokens": toks, "bytes_per_direction": int(per_dir),
            "d2h_gbs": round(per_dir / t_out / 1e9, 2), "h2d_gbs": round(per_dir / t_in / 1e9, 2),
            "link_peak_gbs": link,
            "frac_of_link": {"d2h": round(per_dir / t_out / 1e9 / link["d2h"], 4),
                             "h2d": round(per_dir / t_in / 1e9 / link["h2d"], 4)},
            "link_probe": "contiguous 1 GiB pinned host <-> device cudaMemcpyAsync, best of 6, CUDA events",
            "bit_exact_spot_check": ok, "timing": "host wall clock around issue + wait",
            "overlapped": {"d2h_gbs": round(per_dir / to2 / 1e9, 2), "h2d_gbs": round(per_dir / ti2 / 1e9, 2),
                           "decode_batch": nd, "decode_ms_per_step_alone": round(alone_ms, 4),
                           "decode_ms_per_step_during_swap_out": round(dec_out, 4) if dec_out else None,
                           "decode_ms_per_step_during_swap_in": round(dec_in, 4) if dec_in else None,
                           "decode_steps_during": steps, "staging_bytes": 256 << 20,
                           "why": ("a swap-out makes the compute stream wait until its blocks were read; with "
                                   "staging smaller than the swap each gather first waits for an earlier "
                                   "victim's host copy, so the decode steps follow the host link")},
            "overlapped_whole_swap_staged": {
                "d2h_gbs": round(per_dir / to3 / 1e9, 2), "h2d_gbs": round(per_dir / ti3 / 1e9, 2),
                "decode_ms_per_step_during_swap_out": round(dec_out3, 4) if dec_out3 else None,
                "decode_ms_per_step_during_swap_in": round(dec_in3, 4) if dec_in3 else None,
                "decode_steps_during": steps3, "staging_bytes": int(per_dir)}}


def run_llama(torch, bk, args, device, rank, feed="device", record=0) -> dict:
    """Config 5: random-init Llama-3.2-1B (llm_serving_layer_b200.llama) under
    continuous batching, through forward_varlen with this backend. Requests: a
    final context length from config 2's lognormal (mu = ln 256 - 0.32, sigma =
    0.8, clipped to [16, 2048], mean ~258) and a prompt of lognormal(mu = ln 32
    - 0.32, sigma = 0.8) tokens (at most half the context); Poisson arrivals at
    6 per step, above the completion rate, so the waiting queue never empties.
    Up to 1024 sequences run at once; the initial ones start at a random point
    of their lifetime with synthetic history KV. Each step decodes one token for
    every running sequence past its prompt and prefills at most 512 prompt
    tokens (the reference scheduler's max_prefill_tokens); a waiting request is
    admitted when a slot is free and prefill budget is left. Greedy sampling on
    the GPU (``sample_greedy``, one launch). ``feed="device"``: each sequence's
    last token stays on the GPU (a token per block-table row, written by the
    sampling launch) and the next step's input is assembled there from it and
    the prompt tokens (host scheduling needs only lengths), while the sampled
    tokens travel back asynchronously (``TokenReadback``) and are read one step later,
    so the host never waits for the step it just issued; ``feed="sync"``: the
    step's tokens are read back before the next step is built. ``record``: the
    tokens sampled in the first ``record`` timed steps are returned (for the
    equality check between the two). Each running sequence owns
    a row of DeviceBlockTables (blocks recorded as they are allocated; the
    step's BatchMeta computed on the GPU). Wall clock per step: host scheduling
    and batch assembly, H2D of the step's rows / lengths / new blocks and
    tokens, the 16-layer forward, D2H of the tokens."""
    from llm_serving_layer_b200 import DeviceBlockTables, TokenReadback, sample_greedy
    from llm_serving_layer_b200.llama import LlamaConfig, RandomLlama

    cfg = LlamaConfig()
    model = RandomLlama(cfg, device, seed=args.seed + 17)
    rs = np.random.RandomState(args.seed + 18 + rank)
    n_run, budget, lam = 1024, 512, 6.0

    free = list(rs.permutation(bk.num_blocks))
    bt = DeviceBlockTables(n_run, (2048 + P - 1) // P + 1, P, bk.num_blocks, device=device,
                           max_tokens=n_run + budget, status=bk._status)
    free_rows = list(range(n_run))

    class S:
        __slots__ = ("blocks", "n", "prompt", "pos", "target", "last", "row")
    running, queue = [], []

    def new_req():
        c = int(np.clip(np.round(rs.lognormal(math.log(256) - 0.32, 0.8)), 16, 2048))
        pl = int(np.clip(np.round(rs.lognormal(math.log(32) - 0.32, 0.8)), 4, c // 2))
        r = S()
        r.blocks, r.n, r.prompt, r.pos, r.target = [], 0, rs.randint(0, cfg.vocab, size=pl), 0, c
        r.last = None
        return r

    # initial running set: somewhere inside their lifetime, history KV synthetic
    hist_blocks = []
    for _ in range(n_run):
        r = new_req()
        r.pos = len(r.prompt)
        r.n = int(rs.randint(len(r.prompt), r.target))
        nb = (r.n + P - 1) // P
        r.blocks = [int(free.pop()) for _ in range(nb)]
        hist_blocks += r.blocks
        r.last = int(rs.randint(0, cfg.vocab))
        r.row = free_rows.pop()
        bt.bind(r.row, r.blocks)
        running.append(r)
    idx = torch.tensor(hist_blocks, device=device, dtype=torch.int64)
    g = torch.Generator(device=device).manual_seed(args.seed + 19)
    for layer in range(L):
        for kv in range(2):
            vals = torch.randn((idx.numel(), P, HKV, D), generator=g, device=device) * KV_STD
            bk._pool[layer, kv].index_copy_(0, idx, vals.to(bk.dtype))
            del vals
    for _ in range(256):
        queue.append(new_req())
    # the device-fed loop: each row's last sampled token, on the GPU
    last_dev = torch.zeros(n_run, dtype=torch.int64, device=device)
    init = np.zeros(n_run, dtype=np.int64)
    for r in running:
        init[r.row] = r.last
    last_dev.copy_(torch.from_numpy(init))
    readback = TokenReadback(device)  # sampled tokens of the steps not read back yet
    recorded = []

    def read_back(upto):
        for who, host_tok in readback.collect(upto):
            if who is not None:
                recorded.append(list(zip(who, host_tok.tolist())))

    def step():
        pending = sum(len(r.prompt) - r.pos for r in running if r.pos < len(r.prompt))
        while len(running) < n_run and queue and pending < budget:
            r = queue.pop(0)
            pending += len(r.prompt)
            r.row = free_rows.pop()
            running.append(r)
        left = budget
        batch, qtok = [], []
        for r in running:
            if r.pos < len(r.prompt):
                if left == 0:
                    continue
                take = min(left, len(r.prompt) - r.pos)
                batch.append((r, take))
                qtok.append(r.prompt[r.pos: r.pos + take])
                left -= take
            else:
                batch.append((r, 1))
                qtok.append(np.asarray([r.last]))
        for r, q in batch:
            need = (r.n + q + P - 1) // P - len(r.blocks)
            if need > 0:
                new = [int(free.pop()) for _ in range(need)]
                r.blocks += new
                bt.extend(r.row, new)
            r.n += q
        meta = bt.build_batch_meta([r.row for r, _ in batch], [q for _, q in batch], [r.n for r, _ in batch])
        if feed == "device":
            # one packed transfer: the prompt tokens (0 where a decode row's token goes), the
            # decode rows' token positions and rows, and which entries sample a token into which row
            T = sum(q for _, q in batch)
            dpos, drow, srow = [], [], []
            o = 0
            for j, (r, q) in enumerate(batch):
                if r.pos >= len(r.prompt):
                    dpos.append(o)
                    drow.append(r.row)
                srow.append(r.row if r.pos >= len(r.prompt) or r.pos + q >= len(r.prompt) else -1)
                o += q
            packed = np.concatenate([np.concatenate([t if r.pos < len(r.prompt) else [0]
                                                     for (r, _), t in zip(batch, qtok)]).astype(np.int64),
                                     dpos, drow, srow]).astype(np.int64)
            dev_in = torch.from_numpy(packed).pin_memory().to(device, non_blocking=True)
            nd = len(dpos)
            toks = dev_in[:T].clone()
            toks.index_copy_(0, dev_in[T:T + nd], last_dev.index_select(0, dev_in[T + nd:T + 2 * nd]))
        else:
            toks = torch.from_numpy(np.concatenate(qtok).astype(np.int64)).pin_memory().to(device, non_blocking=True)
        ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        ev[0].record()
        logits = model.forward_varlen(toks, meta, bk)
        ev[1].record()
        fwd_events.append(ev)
        # the entries' identities, the same in both feeds (same seeds, same schedule), while recording
        who = ([(r.row, r.n) for r, _ in batch]
               if counting[0] and len(recorded) + len(readback) < record else None)
        if feed == "device":
            # argmax of every entry's logits, written into its row's token (entries still
            # mid-prompt have row -1 and write nothing), one launch; the tokens travel to the
            # host on a side stream and are read one step later
            sampled = sample_greedy(logits, tokens=last_dev, rows=dev_in[T + 2 * nd:].to(torch.int32),
                                    status=bk._status)
            readback.submit(sampled, who)
            read_back(1)  # the previous step's tokens: streamed one step behind
            nxt = [None] * len(batch)
        else:
            nxt = sample_greedy(logits).cpu().tolist()
            if who is not None:
                recorded.append(list(zip(who, nxt)))
        gen = prompt_tok = 0
        done = []
        for (r, q), t in zip(batch, nxt):
            if r.pos < len(r.prompt):
                r.pos += q
                prompt_tok += q
                if r.pos < len(r.prompt):
                    continue
            r.last = t
            gen += 1
            if r.n + 1 >= r.target:
                done.append(r)
        for r in done:
            running.remove(r)
            free.extend(r.blocks)
            bt.release(r.row)
            free_rows.append(r.row)
        for _ in range(rs.poisson(lam)):
            queue.append(new_req())
        return gen, prompt_tok, len(batch), int(meta.positions.shape[0])

    fwd_events = []
    counting = [False]
    for _ in range(args.warmup):
        step()
    read_back(0)
    torch.cuda.synchronize()
    bk.check_status()
    fwd_events.clear()
    counting[0] = True
    steps = max(20, min(args.llama_steps, 1000))
    gens = prompts = seqs = toks = 0
    t0 = time.perf_counter()
    for _ in range(steps):
        a_, b_, c_, d_ = step()
        gens += a_
        prompts += b_
        seqs += c_
        toks += d_
    read_back(0)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    bk.check_status()
    fwd_ms = sum(a.elapsed_time(b) for a, b in fwd_events) / len(fwd_events)
    del model
    torch.cuda.empty_cache()
    return {"workload": ("config5: random-init Llama-3.2-1B (hidden 2048, 16 layers, 32/8 heads, d 64, FFN 8192, "
                         "vocab 128256, RoPE theta 500000, fp16), continuous batching of up to 1024 sequences, "
                         "final context lognormal mean ~258 cap 2048, prompts lognormal mean ~32, Poisson "
                         "arrivals 6/step, <= 512 prefill tokens per step, greedy"),
            "steps": steps, "generated_tok_per_s": round(gens / dt, 1),
            "processed_tok_per_s": round(toks / dt, 1), "prompt_tok_per_s": round(prompts / dt, 1),
            "ms_per_step": round(dt * 1e3 / steps, 3), "forward_device_ms_per_step": round(fwd_ms, 3),
            "mean_batch_seqs": round(seqs / steps, 1),
            "mean_batch_tokens": round(toks / steps, 1),
            "tokens": recorded,
            "feed": ("last tokens kept on the GPU, next input assembled there, sampled tokens read back "
                     "asynchronously one step later" if feed == "device" else
                     "sampled tokens read back before the next step is built"),
            "attention": ("B200PagedBackend.append_attend(..., rope=): RoPE, KV-append and attention in one "
                          "launch per layer on decode steps; mixed steps: rotation kernel, append, prefill and "
                          "decode kernels"),
            "timing": "host wall clock around the steps (host scheduling, batch assembly, H2D, forward, D2H)"}


def run_flashinfer(args) -> None:
    """The reference's own GPU path on the same B200, as a comparison (not a
    bench line): FlashInfer's BatchDecodeWithPagedKVCacheWrapper(use_tensor_cores
    = False) and BatchPrefillWithPagedKVCacheWrapper (default backend), planned
    once per step and run per layer on (k_pool[l], v_pool[l]) in "NHD" layout
    exactly as the reference configures them
    (serving/backends/flashinfer_backend.py:336-345, 602-676), against this
    package's planned attention on the same pool, page tables and queries:
    config 2's decode steps (16 layers, batch 256) and config 3's prefill steps
    (16 layers), then the large-batch prefill launch (64 chunks of 512 tokens)
    against every FlashInfer paged-prefill backend the wrapper accepts here
    (fa2, trtllm-gen; cuDNN's takes other index conventions and is recorded as
    rejected). Kernel time on the device (CUDA events around each step's 16
    back-to-back attention launches, after the step's plan); the outputs are
    compared. One JSON line."""
    import gc

    import torch

    import flashinfer as fi
    from llm_serving_layer_b200 import B200PagedBackend
    from llm_serving_layer_b200.meta import build_meta

    # the calls here are eager (no graphs): Python's collector, run inside a
    # timed region, would stall the host between two launches of one step
    gc.collect()
    gc.disable()
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    free, total = torch.cuda.mem_get_info(device)
    block_bytes = B200PagedBackend.estimate_pool_bytes(L, 1, P, HKV, D, torch.float16)
    num_blocks = int(min(0.3 * total, free - (16 << 30)) // block_bytes)
    bk = B200PagedBackend(L, num_blocks, P, HKV, HQ, D, device=device, dtype=torch.float16, validate="device")
    rs = np.random.RandomState(args.seed)
    n_steps = 12
    ctx, tables, metas = build_workload(torch, bk, rs, n_steps, device)
    g = torch.Generator(device=device).manual_seed(args.seed)
    qs = [torch.randn((N_SEQ, HQ, D), generator=g, device=device).half() for _ in range(L)]
    ws = [torch.zeros(128 << 20, dtype=torch.uint8, device=device) for _ in range(2)]
    dec = fi.BatchDecodeWithPagedKVCacheWrapper(ws[0], "NHD", use_tensor_cores=False)
    pre = fi.BatchPrefillWithPagedKVCacheWrapper(ws[1], "NHD")
    kv = [(bk.k_pool[l], bk.v_pool[l]) for l in range(L)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(fn):
        e0.record()
        outs = fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3, outs

    def fi_plan_decode(m):
        dec.plan(m.kv_indptr, m.kv_indices, m.kv_last_page_len, HQ, HKV, D, P, pos_encoding_mode="NONE",
                 sm_scale=SCALE, q_data_type=torch.float16, kv_data_type=torch.float16)

    res = {"flashinfer_version": fi.__version__}
    # ---- decode (config 2)
    ours_us, fi_us, diff = [], [], 0.0
    for rep in range(2):
        for m in metas:
            bk.invalidate_plan()
            bk.plan(m)
            torch.cuda.synchronize()
            t, a = timed(lambda: [bk.attend(qs[l], l, SCALE, m) for l in range(L)])
            fi_plan_decode(m)
            torch.cuda.synchronize()
            t2, b = timed(lambda: [dec.run(qs[l], kv[l]) for l in range(L)])
            if rep:
                ours_us.append(t / L)
                fi_us.append(t2 / L)
                diff = max(diff, max(float((x.float() - y.float()).abs().max()) for x, y in zip(a, b)))
    res["decode"] = {"workload": "config 2 decode steps (256 sequences, lognormal ctx mean ~258), 16 layers",
                     "ours_us_per_layer": round(float(np.mean(ours_us)), 2),
                     "flashinfer_us_per_layer": round(float(np.mean(fi_us)), 2),
                     "speedup": round(float(np.mean(fi_us)) / float(np.mean(ours_us)), 2),
                     "max_abs_diff": round(diff, 5),
                     "flashinfer_path": "BatchDecodeWithPagedKVCacheWrapper(use_tensor_cores=False), plan per step"}
    # ---- chunked prefill (config 3)
    work = prefill_workload(args.seed + 3)
    perm = np.random.RandomState(args.seed + 5).permutation(bk.num_blocks)
    remap = {}

    def blk(b):
        if b not in remap:
            remap[b] = int(perm[len(remap)])
        return remap[b]

    ptables = {i: [blk(b) for b in t] for i, t in work["tables"].items()}
    qb = [torch.randn((512, HQ, D), generator=g, device=device).half() for _ in range(L)]
    ours_us, fi_us, diff, steps_used = [], [], 0.0, 0
    for ids, st, en in work["steps"][:: max(1, len(work["steps"]) // 60)]:
        tabs = [ptables[i][:(e + P - 1) // P] for i, e in zip(ids, en)]
        m = build_meta(tabs, en, [e - s for s, e in zip(st, en)], P, device=device)
        T = int(m.positions.shape[0])
        bk.invalidate_plan()
        bk.plan(m)
        pre.plan(m.cu_query_lens, m.kv_indptr, m.kv_indices, m.kv_last_page_len, HQ, HKV, D, P, causal=True,
                 pos_encoding_mode="NONE", sm_scale=SCALE, q_data_type=torch.float16, kv_data_type=torch.float16)
        torch.cuda.synchronize()
        for rep in range(2):
            t, a = timed(lambda: [bk.attend(qb[l][:T], l, SCALE, m) for l in range(L)])
            t2, b = timed(lambda: [pre.run(qb[l][:T], kv[l]) for l in range(L)])
        ours_us.append(t / L)
        fi_us.append(t2 / L)
        diff = max(diff, max(float((x.float() - y.float()).abs().max()) for x, y in zip(a, b)))
        steps_used += 1
    res["prefill"] = {"workload": f"config 3 prefill steps ({steps_used} of {len(work['steps'])}, every "
                                  f"{max(1, len(work['steps']) // 60)}th; <= 512 prompt tokens each), 16 layers",
                      "ours_us_per_layer": round(float(np.mean(ours_us)), 2),
                      "flashinfer_us_per_layer": round(float(np.mean(fi_us)), 2),
                      "speedup": round(float(np.mean(fi_us)) / float(np.mean(ours_us)), 2),
                      "ours_median_us_per_layer": round(float(np.median(ours_us)), 2),
                      "flashinfer_median_us_per_layer": round(float(np.median(fi_us)), 2),
                      "ours_max_us_per_layer": round(float(np.max(ours_us)), 2),
                      "speedup_median": round(float(np.median(fi_us)) / float(np.median(ours_us)), 2),
                      "max_abs_diff": round(diff, 5),
                      "flashinfer_path": "BatchPrefillWithPagedKVCacheWrapper (default backend: fa2 on sm_100), "
                                         "causal, plan per step"}
    # ---- large-batch prefill (the bench's batched_64x512 launch) against each
    # backend FlashInfer offers for paged prefill here, on pages filled with
    # random K/V in all 16 layers (a backend the wrapper rejects is recorded
    # with its message; the rejection comes before any kernel runs)
    m, specs, en, tabs = batched_prefill_case(args, device, perm)
    hist = build_meta(tabs, en, en, P, device=device)
    n_all = int(hist.positions.shape[0])
    for layer in range(L):
        kx = torch.randn((n_all, HKV, D), generator=g, device=device).half()
        vx = torch.randn((n_all, HKV, D), generator=g, device=device).half()
        bk.append_kv(layer, kx, vx, hist)
    del kx, vx
    T = int(m.positions.shape[0])
    qbig = torch.randn((T, HQ, D), generator=g, device=device).half()
    fl, _ = prefill_step_work(None, [s0 for s0, _ in specs], en)
    bk.invalidate_plan()
    bk.plan(m)

    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * 16)]

    def per_launch(fn, reps=16):
        """Median device time of `reps` launches over layers r % 16 (each
        bracketed by its own events, so a host stall between two launches
        lands in no launch's time)."""
        for r in range(3):
            fn(r)
        torch.cuda.synchronize()
        for r in range(reps):
            ev[2 * r].record()
            o = fn(r % L)
            ev[2 * r + 1].record()
        torch.cuda.synchronize()
        return float(np.median([ev[2 * r].elapsed_time(ev[2 * r + 1]) * 1e3 for r in range(reps)])), o

    ours, a = per_launch(lambda l: bk.attend(qbig, l, SCALE, m))
    bk.check_status()
    rb = {"workload": "64 chunks of 512 tokens after cached prefixes of U[64, 512] tokens, one launch "
                      "(bench.py's batched_64x512), fp16, 16 layers' pools",
          "ours_us": round(ours, 1), "ours_tflops": round(fl / ours / 1e6, 1)}
    for name in ("fa2", "cudnn", "trtllm-gen"):
        try:
            w = fi.BatchPrefillWithPagedKVCacheWrapper(ws[1], "NHD", backend=name)
            w.plan(m.cu_query_lens, m.kv_indptr, m.kv_indices, m.kv_last_page_len, HQ, HKV, D, P, causal=True,
                   pos_encoding_mode="NONE", sm_scale=SCALE, q_data_type=torch.float16,
                   kv_data_type=torch.float16)
            t, b = per_launch(lambda l: w.run(qbig, kv[l]))
            rb[name] = {"us": round(t, 1), "tflops": round(fl / t / 1e6, 1), "ours_speedup": round(t / ours, 2),
                        "max_abs_diff": round(float((a.float() - b.float()).abs().max()), 5)}
        except Exception as e:  # a backend this build or box does not offer, or configured otherwise
            rb[name] = {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200] if str(e) else ''}"}
        torch.cuda.synchronize()
    res["prefill_batched"] = rb
    gc.enable()
    res["timing"] = ("CUDA events around each step's 16 back-to-back attention launches, after the step's plan "
                     "(large batch: median of 16 launches over the 16 layers' pools, each between its own "
                     "events, after 3 warm-up launches)")
    print(json.dumps(res), flush=True)


def radix_host(args) -> None:
    """Host time per scheduler step of the block-manager and prefix-cache work
    at 1024 running sequences (config 5's batch): this package's BlockAllocator
    + RadixCache (llm_serving_layer_b200.radix) and, when a reference checkout is
    named by LLM_SERVING_LAYER_REF, the reference's own classes on the same
    operations. Pool of 60 000 16-token blocks; 64 prompt families; before
    timing, published prefixes that no sequence holds fill the rest of the pool
    (as after a long run), so every admission evicts. Each step: every running sequence grows by one token (a block
    when it crosses a page), 6 retire (publish, free), 6 arrive (lookup,
    reserve with eviction, attach, allocate the rest). Reported: median host
    ms per step, with and without the allocator's invariant check after each
    step (the reference's debug mode: a full check; here also the O(1)
    incremental one). One JSON line; CPU only."""
    import importlib
    import os

    def make(mod_alloc, mod_radix, seq_cls):
        return mod_alloc.BlockAllocator, mod_radix.RadixCache, mod_radix.attach_prefix, seq_cls

    class _Seq:
        def __init__(self, alloc, seq_id=0):
            self.alloc, self.seq_id, self.block_size = alloc, seq_id, alloc.block_size
            self.block_ids, self.num_tokens, self.is_freed = [], 0, False

        def blocks_needed_for(self, n):
            return max(0, (self.num_tokens + n + self.block_size - 1) // self.block_size - len(self.block_ids))

        def append(self, n):
            need = self.blocks_needed_for(n)
            if need:
                self.block_ids.extend(self.alloc.allocate(need))
            self.num_tokens += n

        def free(self):
            if not self.is_freed and self.block_ids:
                self.alloc.free(self.block_ids)
            self.block_ids, self.num_tokens, self.is_freed = [], 0, True

    import llm_serving_layer_b200.radix as ours
    impls = {"b200": make(ours, ours, _Seq)}
    ref_root = os.environ.get("LLM_SERVING_LAYER_REF", "")
    if ref_root and Path(ref_root, "serving", "cache", "radix.py").is_file():
        import types
        import llm_serving_layer_b200.meta as meta_mod
        eng = types.ModuleType("engine")
        eng.attention_backend = meta_mod
        sys.modules.setdefault("engine", eng)
        sys.modules.setdefault("engine.attention_backend", meta_mod)
        sys.path.insert(0, ref_root)
        impls["reference"] = make(importlib.import_module("serving.memory.allocator"),
                                  importlib.import_module("serving.cache.radix"), _Seq)

    def run(impl, check: bool, steps: int):
        BA, RC, attach, Seq = impl
        rs = np.random.RandomState(args.seed)
        alloc = BA(num_blocks=60000, block_size=P, watermark_blocks=64)
        cache = RC(alloc)
        fams = [list(rs.randint(0, 32000, size=int(rs.randint(64, 512)))) for _ in range(64)]
        running = []

        def admit():
            f = fams[rs.randint(len(fams))]
            toks = f[: int(rs.randint(16, len(f) + 1))] + list(rs.randint(0, 32000, size=int(rs.randint(16, 200))))
            seq = Seq(alloc)
            res = cache.acquire(toks)
            if res.block_ids:
                attach(seq, res.block_ids, res.n_tokens)
            cache.reserve(seq.blocks_needed_for(len(toks) - res.n_tokens), watermark=False)
            seq.append(len(toks) - res.n_tokens)
            running.append([seq, toks, int(rs.randint(16, 400))])

        while len(running) < 1024:
            admit()
        # the cache fills the rest of the pool with published, unused prefixes (as after a
        # long run), so every admission below has to evict
        while alloc.num_free > 200:
            f = fams[rs.randint(len(fams))]
            toks = f[: int(rs.randint(16, len(f) + 1))] + list(rs.randint(0, 32000, size=int(rs.randint(16, 200))))
            seq = Seq(alloc)
            seq.append(min(len(toks), P * (alloc.num_free - 100)))
            cache.insert(toks[: seq.num_tokens], seq.block_ids)
            seq.free()
        times = []
        for st in range(steps):
            t0 = time.perf_counter()
            for r in running:  # one token each; a new block when a page fills
                if r[0].blocks_needed_for(1):
                    cache.reserve(1, watermark=False)
                r[0].append(1)
                r[1].append(7)
                r[2] -= 1
            for _ in range(6):  # retire: publish, then free
                i = max(range(len(running)), key=lambda j: -running[j][2]) if st % 2 else rs.randint(len(running))
                seq, toks, _ = running.pop(i)
                cache.insert(toks[: seq.num_tokens], seq.block_ids)
                seq.free()
            for _ in range(6):
                admit()
            if check == "full":
                alloc.check_invariants()
            elif check == "incremental":
                alloc.check_invariants(full=False)
            times.append(time.perf_counter() - t0)
        return {"ms_per_step_median": round(1e3 * statistics.median(times[2:]), 3),
                "cached_blocks": cache.cached_blocks, "evictions": cache.stats.evictions,
                "free_blocks": alloc.num_free}

    out = {"workload": ("block manager + radix prefix cache host work per scheduler step at 1024 running "
                        "sequences: 60000 16-token blocks (the rest of the pool held by cached prefixes), 64 prompt families, 6 arrivals and 6 retirements "
                        "per step, every sequence +1 token"), "steps": args.radix_steps}
    for name, impl in impls.items():
        out[name] = {"no_check": run(impl, None, args.radix_steps),
                     "full_check_every_step": run(impl, "full", args.radix_steps)}
        if name == "b200":
            out[name]["incremental_check_every_step"] = run(impl, "incremental", args.radix_steps)
    if "reference" not in impls:
        out["reference"] = "not run: set LLM_SERVING_LAYER_REF to a reference checkout to time its classes beside"
    print(json.dumps(out), flush=True)


def decode_sweep() -> None:
    """The decode kernel against batch size: for 64-2048 sequences with config
    2's context distribution (scattered pages of a pool sized for the largest
    batch), one graph of the 16 layers' decode launches back to back, replayed
    20 times after 3 warm-up replays; per launch, the mean time and the
    algorithmic bytes (K and V rows, q and out, page descriptors) over it as a
    fraction of the measured HBM peak. The 16 layers' K/V (≥ 0.5 GB per replay
    at 64 sequences) exceed L2. One JSON line per batch size."""
    import torch

    from llm_serving_layer_b200 import B200PagedBackend
    from llm_serving_layer_b200.meta import build_meta

    dev = torch.device("cuda", 0)
    sizes = (64, 128, 256, 512, 1024, 2048)
    rs = np.random.RandomState(2026)
    ctxs = {n: contexts(rs, n) for n in sizes}
    nb = int(max(((c + P - 1) // P).sum() for c in ctxs.values())) + 64
    bk = B200PagedBackend(L, nb, P, HKV, HQ, D, device=dev, dtype=torch.float16, validate="device")
    g = torch.Generator(device=dev).manual_seed(7)
    for layer in range(L):
        for kv in range(2):
            bk._pool[layer, kv].normal_(0.0, KV_STD, generator=g)
    peak, peak_kind = measured_peaks()
    for n in sizes:
        ctx = ctxs[n]
        perm = rs.permutation(nb)
        tables, o = [], 0
        for c in ctx:
            k = int((c + P - 1) // P)
            tables.append(perm[o:o + k].tolist())
            o += k
        m = build_meta(tables, ctx, [1] * n, P, device=dev)
        q = torch.randn((n, HQ, D), generator=g, device=dev).half()
        out = torch.empty_like(q)
        bk.invalidate_plan()
        bk.reserve_workspace(n, o)
        bk.plan(m)
        for layer in range(L):
            bk.attend(q, layer, SCALE, m, out=out)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for layer in range(L):
                bk.attend(q, layer, SCALE, m, out=out)
        for _ in range(3):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(20):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        bk.check_status()
        us = e0.elapsed_time(e1) * 1e3 / (20 * L)
        alg = int(ctx.sum()) * HKV * D * 2 * 2 + n * HQ * D * 2 * 2 + o * 8
        print(json.dumps({"decode_sweep": {"n_seqs": n, "pages": o, "avg_launch_us": round(us, 2),
                                           "alg_bytes_per_launch": alg,
                                           "achieved_gbs": round(alg / us / 1e3, 1), "peak_gbs": peak,
                                           "peak_kind": peak_kind, "frac": round(alg / us / 1e3 / peak, 4)}}),
              flush=True)
        del graph


def kvops_probe() -> None:
    """A small fixed workload of the KV-append, copy-on-write and swap kernels
    for kernel profilers (ncu): on a 16-layer, 8000-block (4 GB) pool,
    append_kv of 256 scattered slots per layer (config 2's step) 3 x 16 times,
    copy_blocks of 420 pairs (config 3's copy-on-write count) 3 times, and
    swap_out + swap_in of 8 victims x 64 blocks twice. Prints one JSON line."""
    import torch

    from llm_serving_layer_b200 import B200PagedBackend, B200SwapSpace
    from llm_serving_layer_b200.meta import BatchMeta

    dev = torch.device("cuda", 0)
    nb = 8000
    bk = B200PagedBackend(L, nb, P, HKV, HQ, D, device=dev, dtype=torch.float16, validate="device")
    rs = np.random.RandomState(0)
    perm = rs.permutation(nb)
    slots = torch.as_tensor(perm[:256] * P + rs.randint(0, P, 256), dtype=torch.int32, device=dev)
    z = torch.zeros(1, dtype=torch.int32, device=dev)
    m = BatchMeta(query_lens=z, cu_query_lens=torch.zeros(2, dtype=torch.int32, device=dev), kv_lens=z,
                  positions=torch.zeros(256, dtype=torch.int64, device=dev), last_token_ix=z,
                  kv_indptr=torch.zeros(2, dtype=torch.int32, device=dev),
                  kv_indices=torch.zeros(0, dtype=torch.int32, device=dev), kv_last_page_len=z,
                  batch_indices=torch.zeros(256, dtype=torch.int32, device=dev), slot_mapping=slots)
    k = torch.randn(256, HKV, D, device=dev).half()
    v = torch.randn(256, HKV, D, device=dev).half()
    for _ in range(3):
        for layer in range(L):
            bk.append_kv(layer, k, v, m)
    src, dst = perm[256:676].tolist(), perm[676:1096].tolist()
    for _ in range(3):
        bk.copy_blocks(src, dst)
    sw = B200SwapSpace(bk, staging_bytes=512 << 20, synchronous=True)

    class Blocks:
        def __init__(self, ids, n):
            self.block_ids, self.num_tokens, self.seq_id, self.is_freed = list(ids), n, 0, False

    vic = [perm[1100 + 64 * i:1164 + 64 * i].tolist() for i in range(8)]
    new = [perm[1700 + 64 * i:1764 + 64 * i].tolist() for i in range(8)]
    for _ in range(2):
        hs = [sw.swap_out(f"v{i}", Blocks(vic[i], 1024)) for i in range(8)]
        for i in range(8):
            sw.swap_in(hs[i], Blocks(new[i], 1024))
        for h in hs:
            sw.release(h)
    torch.cuda.synchronize()
    bk.check_status()
    print(json.dumps({"kvops_probe": "ok", "appends": 3 * L, "copy_blocks_launches": 3, "swaps": 16}))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--seed", type=int, default=2026)
    ap.add_argument("--pool-frac", type=float, default=0.9)
    ap.add_argument("--max-graphs", type=int, default=32)
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU oracle timing (0 = skip)")
    ap.add_argument("--no-swap", dest="swap", action="store_false")
    ap.add_argument("--no-prefill", dest="prefill", action="store_false")
    ap.add_argument("--no-llama", dest="llama", action="store_false")
    ap.add_argument("--fused", dest="fuse", action="store_true",
                    help="time the fused append_attend step as the main value (default: append_kv + attend, "
                         "the reference API, with the fused step reported beside it)")
    ap.add_argument("--no-fused-extra", dest="fused_extra", action="store_false")
    ap.add_argument("--llama-steps", type=int, default=100)
    ap.add_argument("--kvops-probe", action="store_true",
                    help="run only the small append / copy-on-write / swap workload (for kernel profilers)")
    ap.add_argument("--radix-host", action="store_true",
                    help="CPU only: host time per step of the block allocator and radix cache at 1024 sequences")
    ap.add_argument("--radix-steps", type=int, default=40)
    ap.add_argument("--flashinfer", action="store_true",
                    help="compare against FlashInfer (the reference's GPU backend) on config 2 and 3 inputs")
    ap.add_argument("--decode-sweep", action="store_true",
                    help="run only the decode kernel over batch sizes 64-2048 (one JSON line per size)")
    args = ap.parse_args()
    if args.kvops_probe:
        kvops_probe()
        return
    if args.decode_sweep:
        decode_sweep()
        return
    if args.flashinfer:
        run_flashinfer(args)
        return
    if args.radix_host:
        radix_host(args)
        return
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        args.steps_ref = max(1, min(args.steps, 100))
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
