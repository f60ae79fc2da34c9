"""Verify-step benchmark (tree build + tree verify attention + acceptance), B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mfd|reference] [--requests R]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU; the driver's launch)
    python bench.py --config C                             (one BASELINE config's kernels alone, C = 0..3)
    python bench.py --north-star                           (the north-star step alone: batch 1, greedy)
    python bench.py --kernel K                             (one kernel alone, L2 flushed between launches: a kernel
                                                            of the batch step -- logits_step, tree_build, attention,
                                                            accept --, of the commit step -- commit_kv, gdn_commit --,
                                                            or the paged drafter attention, paged_mode_attn)

Workload (synthetic, seeded per global request id so any partition computes the same
requests): 256 requests per step, partitioned 256/128/64/32 per GPU at 1/2/4/8 GPUs (strong scaling: the job is
fixed, the GPUs share it).  Each request has drafter logits float32 [K=8, L=16, V=151936] (N(0,1), 4 ids per
(mode, position) boosted by U(4,10)), an exact mixture tree of B=64 nodes, tree-masked GQA verify attention (32/8
heads, head_dim 128, prefix U(1024, 8192)), and stochastic acceptance at T=1 over target logits bf16 [65, V]
N(0, 1.5) with seeded uniforms.  Requests are partitioned across ranks (sorted by prefix, dealt round-robin); there
is no collective on the data path (only the timing max-reduce).  Inputs (~117 MB per request, 30 GB per step at
one GPU) are far larger than L2.

Printed by rank 0: one JSON line (metric trees/s, whole job), with
  north_star:    BASELINE's headline verify step -- batch 1, greedy, prefix 4096, configs 0 + 1 + acceptance --
                 in microseconds per step (L2 flushed between steps), rank 0 only;
  roofline:      the dominant kernel (the fused logits step) against the measured HBM copy bandwidth;
  step_roofline: the whole step's algorithmic bytes against the same peak;
  e2e:           the same metric through the public API with inputs copied from pinned host memory each step;
  cpu_baseline:  the reference's CPU path (its compiled C++ builder, torch's CPU top-k / logsumexp / SDPA /
                 softmax sampling, its walk) on a bounded sample, compute only, rank 0 at N=1.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

K_MODES, L_BLOCK, VOCAB, BUDGET = 8, 16, 151936, 64
W = BUDGET + 1
H, HKV, D = 32, 8, 128
TOTAL_REQUESTS = 256     # 256 requests, partitioned 256/128/64/32 per GPU at 1/2/4/8 GPUs
REQUESTS_PER_GPU = 32    # the --kernel / --config profiling cases
# Logits-step DRAM traffic per row (read + write) from an ncu capture of 1024 rows x 151936 fp32, k = 64
# (bench.py --kernel logits_step --requests-per-gpu 8): 622.52 MB read + 4.65 MB written.  Traffic grows with the
# rows, so a launch of R rows moves R times this.
TOPK_TRAFFIC_PER_ROW = (622.516224e6 + 4.645376e6) / 1024
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


# ------------------------------------------------------------------------------------------------ setup

def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]), "source": "measured"}
    except Exception:
        return dict(PEAKS_FALLBACK, source="fallback")


def dist_setup(n_gpus: int):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        torch.cuda.set_device(local)
        # a short timeout: a rank that fails ends the others' next collective with an error instead of a hang
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()


def max_over_ranks(ws, value: float) -> float:
    if ws == 1:
        return value
    dev = "cuda" if torch.distributed.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(ws, value: float) -> float:
    if ws == 1:
        return value
    dev = "cuda" if torch.distributed.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.SUM)
    return float(t.item())


def prefix_lengths(total: int, seed: int = 4321):
    """Prefix length of every request id: U(1024, 8192), the same for a request whatever the job size."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(1024, 8193, (max(total, 256),), generator=g).tolist()[:total]


def partition(total: int, ws: int, rank: int, prefixes):
    """This rank's request ids: sorted by prefix length and dealt round-robin, so every rank gets the same count
    and nearly the same attention work."""
    order = sorted(range(total), key=lambda r: prefixes[r])
    return order[rank::ws]


def gen_draft_logits(req: int, dev, out: torch.Tensor):
    g = torch.Generator(device=dev).manual_seed(1_000_003 * (req + 1))
    out.normal_(generator=g)
    ids = torch.randint(0, VOCAB, (K_MODES, L_BLOCK, 4), generator=g, device=dev)
    boost = torch.rand(K_MODES, L_BLOCK, 4, generator=g, device=dev) * 6 + 4
    out.scatter_add_(2, ids, boost)


def sharp_draft_logits(seed: int, dev, out: torch.Tensor, share: float = 0.75):
    """configs[3]'s drafter logits [K, L, V] float32: N(0,1) plus, per (mode, position), one token boosted by
    U(12, 16) -- the position's consensus token for a mode with probability `share`, else a token of the mode's
    own.  The modes then share a deep chain and branch off it, so a B=64 mixture tree reaches depth 9 and more
    (the config-0 generator's trees are about 3 deep)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    out.normal_(generator=g)
    consensus = torch.randint(0, VOCAB, (1, L_BLOCK, 1), generator=g, device=dev).expand(K_MODES, L_BLOCK, 1)
    own = torch.randint(0, VOCAB, (K_MODES, L_BLOCK, 1), generator=g, device=dev)
    pick = torch.rand(K_MODES, L_BLOCK, 1, generator=g, device=dev) < share
    ids = torch.where(pick, consensus, own)
    out.scatter_add_(2, ids, torch.rand(K_MODES, L_BLOCK, 1, generator=g, device=dev) * 4 + 12)


def forced_path(tokens, parents, depths, depth: int, seed: int):
    """A seeded random root-to-node path of `depth` edges in one tree (tokens/parents/depths: host sequences of the
    W verify rows, node 0 the root; depths[0] = 0).  Picks uniformly among the nodes at that depth, preferring
    leaves; returns the node ids root..end, or the deepest available path when the tree is shallower."""
    n = len(parents)
    has_child = [False] * n
    for i in range(1, n):
        if parents[i] >= 0:
            has_child[parents[i]] = True
    real = [i for i in range(n) if i == 0 or parents[i] >= 0]
    depth = min(depth, max(depths[i] for i in real))
    at = [i for i in real if depths[i] == depth]
    leaves = [i for i in at if not has_child[i]]
    pool = leaves or at
    g = torch.Generator().manual_seed(seed)
    end = pool[int(torch.randint(0, len(pool), (1,), generator=g))]
    path = [end]
    while path[-1] != 0:
        path.append(parents[path[-1]])
    return path[::-1]


def force_argmax(target: torch.Tensor, tokens, path):
    """target [W, V] logits: along the path, each node's row gets its argmax forced onto the next path node's token
    (value = the row's maximum + 1), so the greedy walk accepts exactly the path (the last node's row keeps its own
    argmax, the bonus token)."""
    for a, b in zip(path[:-1], path[1:]):
        row = target[a]
        row[int(tokens[b])] = row.float().max() + 1.0


class Batch:
    """Device-resident inputs and outputs of one rank's requests."""

    def __init__(self, reqs, prefixes, dev, temperature=1.0, target_std=1.5, uniform_prefix=None):
        self.reqs = reqs
        bs = len(reqs)
        self.bs = bs
        self.temperature = temperature
        self.prefix = [uniform_prefix or prefixes[r] for r in reqs]
        smax = max(self.prefix) + W
        self.draft = torch.empty(bs, K_MODES, L_BLOCK, VOCAB, dtype=torch.float32, device=dev)
        self.q = torch.empty(bs, W, H, D, dtype=torch.bfloat16, device=dev)
        self.k = torch.empty(bs, HKV, smax, D, dtype=torch.bfloat16, device=dev)
        self.v = torch.empty(bs, HKV, smax, D, dtype=torch.bfloat16, device=dev)
        self.target = torch.empty(bs, W, VOCAB, dtype=torch.bfloat16, device=dev)
        self.u = torch.empty(bs, W, dtype=torch.float64, device=dev)
        for i, r in enumerate(reqs):
            gen_draft_logits(r, dev, self.draft[i])
            g = torch.Generator(device=dev).manual_seed(7_000_001 * (r + 1))
            self.q[i].copy_(torch.randn(W, H, D, generator=g, device=dev))
            # each request's keys are drawn at its own length (prefix + tree), so its values do not depend on the
            # other requests of the batch (the padding beyond prefix + W is never read)
            p = self.prefix[i]
            self.k[i, :, :p + W].copy_(torch.randn(HKV, p + W, D, generator=g, device=dev) * 0.5)
            self.v[i, :, :p + W].copy_(torch.randn(HKV, p + W, D, generator=g, device=dev) * 0.5)
            self.target[i].copy_(torch.randn(W, VOCAB, generator=g, device=dev) * target_std)
            self.u[i].copy_(torch.rand(W, generator=g, device=dev, dtype=torch.float64))
        self.prefix_t = torch.tensor(self.prefix, dtype=torch.int32, device=dev)
        # outputs / intermediates
        R = bs * K_MODES * L_BLOCK
        self.top = torch.empty(R, BUDGET, dtype=torch.float32, device=dev)
        self.ids = torch.empty(R, BUDGET, dtype=torch.int32, device=dev)
        self.logz = torch.empty(R, dtype=torch.float32, device=dev)
        self.tree = torch.empty(bs, 3, W, dtype=torch.int64, device=dev)
        self.counts = torch.empty(bs, dtype=torch.int64, device=dev)
        self.attn_out = torch.empty(bs, W, H, D, dtype=torch.bfloat16, device=dev)

    def input_bytes(self):
        kv = sum(2 * HKV * (p + W) * D * 2 for p in self.prefix)
        return self.draft.numel() * 4 + self.q.numel() * 2 + kv + self.target.numel() * 2 + self.u.numel() * 8

    def step_bytes(self):
        """Algorithmic bytes of one step: the inputs read once, the logits-step results (top log-probs, ids, log Z)
        written once and read back by the tree build, the trees, the attention output and the accept outputs."""
        cand = self.top.numel() * 4 + self.ids.numel() * 4 + self.logz.numel() * 4
        return (self.input_bytes() + 2 * cand + self.tree.numel() * 8 + self.attn_out.numel() * 2
                + self.bs * (W * 8 + 3 * L_BLOCK * 8 + 32))


# ------------------------------------------------------------------------------------------------ the step

class Step:
    """One verify step over a Batch: 4 kernel launches (logits step, tree build, attention, accept)."""

    LAUNCHES = 4

    def __init__(self, batch: Batch, splits=None):
        from mfd_b200 import ops

        self.ops = ops
        self.b = batch
        self.splits = splits or ops.default_splits(batch.bs, W, H, HKV, batch.k.shape[2])

    def run(self, ev=None):
        b, ops = self.b, self.ops
        if ev is not None:
            ev[0].record()
        ops.topk_logz(b.draft.view(-1, VOCAB), BUDGET, ids_dtype=torch.int32, out=(b.top, b.ids, b.logz))
        if ev is not None:
            ev[1].record()
        _, _, anc, _ = ops.build_trees(b.top.view(b.bs, K_MODES, L_BLOCK, BUDGET),
                                       b.ids.view(b.bs, K_MODES, L_BLOCK, BUDGET), None, BUDGET, tree=b.tree,
                                       counts=b.counts)
        if ev is not None:
            ev[2].record()
        ops.tree_attention(b.q, b.k, b.v, anc, b.prefix_t, D ** -0.5, splits=self.splits, out=b.attn_out)
        if ev is not None:
            ev[3].record()
        o = ops.accept(b.target, b.tree[:, 0], b.tree[:, 2], temperature=b.temperature,
                       uniforms=b.u if b.temperature > 0 else None, max_steps=L_BLOCK - 1, out_len=L_BLOCK)
        if ev is not None:
            ev[4].record()
        return o


# ------------------------------------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi sampling SM clocks and throttle reasons every 200 ms, started (one fork) before the timed region
    and stopped after it, so that no process is spawned while kernels are being launched."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._proc = None

    def __enter__(self):
        try:
            self._proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                           "--format=csv,noheader,nounits", "-lms", "200"],
                                          stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.5)  # let the first sample land before timing starts
        except Exception:
            self._proc = None
        return self

    def __exit__(self, *a):
        if self._proc is None:
            return
        time.sleep(0.25)  # one more sample after the timed region
        self._proc.terminate()
        try:
            out, _ = self._proc.communicate(timeout=10)
        except Exception:
            self._proc.kill()
            out, _ = self._proc.communicate()
        for line in out.splitlines():
            vals = [v.strip() for v in line.split(",")]
            if len(vals) == 7:
                self.samples.append(vals)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------------ measurements

def time_steps(step: Step, steps: int, warmup: int, ws: int, dev_index: int):
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev_index) as clocks:  # sampling spans the warm-up and the timed steps
        for _ in range(warmup):
            step.run()
        barrier(ws)
        start.record()
        for i in range(steps):
            step.run(evs[i])
        end.record()
        torch.cuda.synchronize()
    barrier(ws)
    total_ms = start.elapsed_time(end)
    per_kernel = {name: statistics.mean(e[j].elapsed_time(e[j + 1]) for e in evs) * 1e3
                  for j, name in enumerate(["logits_step", "tree_build", "attention", "accept"])}
    return total_ms, per_kernel, clocks.summary()


def north_star(dev, steps: int, warmup: int, graph: bool = True):
    """Batch 1, greedy, prefix 4096: BASELINE's headline verify step; L2 flushed between timed steps."""
    prefixes = [4096]
    batch = Batch([0], prefixes, dev, temperature=0.0, target_std=1.0, uniform_prefix=4096)
    step = Step(batch)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(max(warmup, 3)):
        step.run()
    times, parts = [], {"logits_step": [], "tree_build": [], "attention": [], "accept": []}
    for _ in range(steps):
        flush.zero_()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        step.run(ev)
        torch.cuda.synchronize()
        times.append(ev[0].elapsed_time(ev[4]) * 1e3)
        for j, name in enumerate(parts):
            parts[name].append(ev[j].elapsed_time(ev[j + 1]) * 1e3)
    # the same four launches captured once in a CUDA graph and replayed (as a serving loop would run them): the
    # replay has no host launch gaps between the kernels, which the eager step above can have
    graph_times = []
    if graph:  # (single-process runs only: under torchrun the process group's threads share the device)
        try:
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                step.run()
            for _ in range(max(warmup, 3)):
                g.replay()
            for _ in range(steps):
                flush.zero_()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda._sleep(2_000_000)
                s.record()
                g.replay()
                e.record()
                torch.cuda.synchronize()
                graph_times.append(s.elapsed_time(e) * 1e3)
            del g
        except RuntimeError as exc:  # capture refused: report the eager step only
            print(f"north_star: CUDA graph capture failed ({exc}); eager step only", file=sys.stderr)
    alg_bytes = batch.input_bytes()
    us_eager = statistics.mean(times)
    us = statistics.mean(graph_times) if graph_times else us_eager
    pk = peaks()
    roof_us = alg_bytes / (pk["hbm_gbs"] * 1e9) * 1e6
    return {
        "us_per_step": round(us, 2), "how": "CUDA graph replay" if graph_times else "eager launches",
        "us_eager": round(us_eager, 2), "us_eager_median": round(statistics.median(times), 2),
        "parts_us": {k: round(statistics.mean(v), 2) for k, v in parts.items()},
        "algorithmic_bytes": alg_bytes, "roofline_us": round(roof_us, 2),
        "frac_of_hbm_roofline": round(roof_us / us, 4),
        "config": "batch 1, K=8 L=16 V=151936 fp32 draft logits, B=64, prefix 4096, 32/8 heads d128, greedy",
        "l2": "flushed (256 MB write) before every timed step",
    }


def h2d_link_gbs(dev, nbytes: int = 1 << 30, reps: int = 5) -> float:
    """Pinned host -> device copy bandwidth of this GPU's link (best of `reps` copies of 1 GiB, CUDA events)."""
    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    dst.copy_(src, non_blocking=True)
    best = float("inf")
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        dst.copy_(src, non_blocking=True)
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e))
    del src, dst
    return nbytes / (best * 1e-3) / 1e9


E2E_FIELDS = ("draft", "q", "k", "v", "target", "u", "prefix_t")


def e2e(dev, reqs, prefixes, steps: int, ws: int, sample: int = 16, chunk: int = 4):
    """The public API end to end on every rank, over a sample of its requests: each step copies those requests'
    inputs from pinned host memory to the device (a copy stream, `chunk` requests at a time, so the copy of one
    chunk overlaps the verify step of the previous one), runs the verify step per chunk, and reads the accepted
    lengths, accepted tokens and trees back into pinned host memory.  Timed on the device (CUDA events), max over
    ranks; value = requests of all ranks per second.  The copies dominate: the drafter logits alone are 77.8 MB
    per request, so the line also reports the H2D rate against this link's measured pinned-copy bandwidth."""
    sample_reqs = reqs[:sample]
    groups = [sample_reqs[i:i + chunk] for i in range(0, len(sample_reqs), chunk)]
    batches = [Batch(g, prefixes, dev) for g in groups]
    hosts = [{name: getattr(b, name).cpu().pin_memory() for name in E2E_FIELDS} for b in batches]
    steps_ = [Step(b) for b in batches]
    outs = [(torch.empty(b.bs, dtype=torch.int32).pin_memory(), torch.empty(b.bs, L_BLOCK, dtype=torch.int64).pin_memory(),
             torch.empty_like(b.tree, device="cpu").pin_memory()) for b in batches]
    h2d = sum(t.numel() * t.element_size() for h in hosts for t in h.values())
    d2h = sum(t.numel() * t.element_size() for o in outs for t in o)
    cur = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    done = [torch.cuda.Event() for _ in batches]
    ready = [torch.cuda.Event() for _ in batches]
    for ev in done:
        ev.record(cur)

    def one():
        for j, (b, h, st, o) in enumerate(zip(batches, hosts, steps_, outs)):
            with torch.cuda.stream(copy):
                copy.wait_event(done[j])  # this chunk's buffers are free once its previous step has read them
                for name, t in h.items():
                    getattr(b, name).copy_(t, non_blocking=True)
                ready[j].record(copy)
            cur.wait_event(ready[j])
            r = st.run()
            o[0].copy_(r["accept_len"], non_blocking=True)
            o[1].copy_(r["out_tokens"], non_blocking=True)
            o[2].copy_(b.tree, non_blocking=True)
            done[j].record(cur)

    one()
    torch.cuda.synchronize()
    barrier(ws)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(cur)
    copy.wait_event(s)
    for _ in range(steps):
        one()
    e.record(cur)
    torch.cuda.synchronize()
    ms = max_over_ranks(ws, s.elapsed_time(e) / steps)
    assert all(int(o[0].min()) >= 0 for o in outs)  # the results were read back
    link = h2d_link_gbs(dev)
    rate = h2d / (ms * 1e-3) / 1e9
    del batches, steps_, hosts
    return {"value": round(len(sample_reqs) * ws / (ms / 1e3), 3), "unit": "trees/s",
            "h2d_bytes_per_step": h2d * ws, "d2h_bytes_per_step": d2h * ws,
            "requests_per_step": len(sample_reqs) * ws, "ms_per_step": round(ms, 3),
            "h2d_gbs_per_gpu": round(rate, 1), "h2d_link_gbs_measured": round(link, 1),
            "h2d_frac_of_link": round(rate / link, 4),
            "bound": "host-to-device copies (PCIe): the step's inputs cross the link once per step",
            "how": f"{len(sample_reqs)} requests per GPU from pinned host memory in chunks of {chunk}, copy stream "
                   "overlapped with the previous chunk's verify step; results read back to pinned memory"}


def commit_line(name: str, steps: int, warmup: int, requests: int):
    """The commit step's kernels alone (synthetic stand-ins of a hybrid target; L2 flushed per launch):
      commit_kv  -- token-major pool moves: `requests` requests x 16-wide move lists with 8 accepted moves each,
                    32 buffers (K and V of 16 attention layers) of 2 KB slots (8 KV heads x 128 x bf16);
      gdn_commit -- 36 GDN layers, states [32, 128, 128] float32, an 8-node accepted path of a 65-node tree, plus
                    the conv windows [6144, 4] bf16 (mfd_conv_commit)."""
    from mfd_b200 import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(5)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    if name == "commit_kv":
        width, moves, nbuf, slot = 16, 8, 32, 2048
        per_req = 80
        slots = requests * per_req
        bufs = [torch.empty(slots, slot // 2, dtype=torch.bfloat16, device=dev).normal_(generator=g) for _ in range(nbuf)]
        src = torch.zeros(requests, width, dtype=torch.int64)
        tgt = torch.zeros(requests, width, dtype=torch.int64)
        for b in range(requests):
            base = b * per_req
            for i in range(moves):
                src[b, i], tgt[b, i] = base + 10 + 2 * i + 1, base + 10 + i  # node slot -> position slot
        src, tgt = src.to(dev), tgt.to(dev)
        ptrs = torch.tensor([t.data_ptr() for t in bufs], dtype=torch.int64, device=dev)
        us = timed_us(lambda: ops.commit_kv_moves(ptrs, slot, src, tgt, base_align=16, pool_slots=slots), steps, warmup,
                     flush)
        alg = requests * moves * nbuf * slot * 2
        work = f"{requests} requests x {moves} moves x {nbuf} buffers x {slot} B slots"
    else:
        layers, H, HK, D, n, plen, conv_dim, kernel = 36, 32, 16, 128, 65, 8, 6144, 4
        states = [torch.empty(H, D, D, device=dev).normal_(generator=g) for _ in range(layers)]
        us_ = [torch.empty(n, H, D, device=dev).normal_(generator=g) for _ in range(layers)]
        ks = [torch.empty(n, HK, D, device=dev).normal_(generator=g).bfloat16() for _ in range(layers)]
        gs = [torch.empty(n, H, device=dev).uniform_(-2, 0, generator=g) for _ in range(layers)]
        convs = [torch.empty(conv_dim, kernel, device=dev).normal_(generator=g).bfloat16() for _ in range(layers)]
        xs = [torch.empty(n, conv_dim, device=dev).normal_(generator=g).bfloat16() for _ in range(layers)]
        path = torch.tensor([0, 1, 3, 7, 12, 20, 31, 40], dtype=torch.int64, device=dev)
        window = torch.tensor([kernel + 12, kernel + 20, kernel + 31, kernel + 40], dtype=torch.int32, device=dev)

        def fn():
            ops.gdn_commit(states, us_, ks, gs, path)
            ops.conv_commit(convs, xs, window)

        us = timed_us(fn, steps, warmup, flush)
        alg = layers * (H * D * D * 4 * 2 + plen * (H * D * 4 + HK * D * 2) + conv_dim * kernel * 2 * 2)
        work = f"{layers} GDN layers x [{H}, {D}, {D}] f32 states, {plen}-node path, conv [{conv_dim}, {kernel}] bf16"
    return {"kernel": name, "workload": work, "us_per_launch": round(us, 2), "algorithmic_bytes": alg,
            "achieved_gbs": round(alg / us / 1e3, 1), "peak_hbm_gbs": peaks()["hbm_gbs"],
            "frac_of_hbm": round(alg / us / 1e3 / peaks()["hbm_gbs"], 4), "l2": "flushed (256 MB write) per launch"}


def kernel_line(name: str, steps: int, warmup: int, requests: int):
    """One kernel of the batch step alone, on the batch workload of one GPU (the profiling case of its ncu
    summaries): device time per launch with the L2 flushed (256 MB write) before each."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    prefixes = prefix_lengths(requests)
    batch = Batch(list(range(requests)), prefixes, dev)
    step = Step(batch)
    step.run()  # the trees and ancestor bitsets the later kernels read
    ops, b = step.ops, batch
    _, _, anc, _ = ops.build_trees(b.top.view(b.bs, K_MODES, L_BLOCK, BUDGET), b.ids.view(b.bs, K_MODES, L_BLOCK, BUDGET),
                                   None, BUDGET, tree=b.tree, counts=b.counts)
    fns = {
        "logits_step": lambda: ops.topk_logz(b.draft.view(-1, VOCAB), BUDGET, ids_dtype=torch.int32,
                                             out=(b.top, b.ids, b.logz)),
        "tree_build": lambda: ops.build_trees(b.top.view(b.bs, K_MODES, L_BLOCK, BUDGET),
                                              b.ids.view(b.bs, K_MODES, L_BLOCK, BUDGET), None, BUDGET, tree=b.tree,
                                              counts=b.counts),
        "attention": lambda: ops.tree_attention(b.q, b.k, b.v, anc, b.prefix_t, D ** -0.5, splits=step.splits,
                                                out=b.attn_out),
        "accept": lambda: ops.accept(b.target, b.tree[:, 0], b.tree[:, 2], temperature=b.temperature, uniforms=b.u,
                                     max_steps=L_BLOCK - 1, out_len=L_BLOCK),
    }
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    us = timed_us(fns[name], steps, warmup, flush)
    rows = requests * K_MODES * L_BLOCK
    alg = {"logits_step": rows * VOCAB * 4, "tree_build": rows * BUDGET * 8,
           "attention": sum(2 * HKV * (p + W) * D * 2 for p in batch.prefix) + b.q.numel() * 2 * 2,
           "accept": b.target.numel() * 2}[name]
    return {"kernel": name, "requests": requests, "us_per_launch": round(us, 2), "algorithmic_bytes": alg,
            "achieved_gbs": round(alg / us / 1e3, 1), "peak_hbm_gbs": peaks()["hbm_gbs"],
            "frac_of_hbm": round(alg / us / 1e3 / peaks()["hbm_gbs"], 4), "l2": "flushed (256 MB write) per launch"}


def paged_line(steps: int, warmup: int, requests: int):
    """The SGLang paged mode attention of one draft layer for a serving batch: `requests` requests, K = 8 modes of
    16-token blocks (128 queries x 32 heads each), contexts U(1024, 8192) held in a paged KV cache [slots, 8, 128]
    whose slots are a random permutation (req_to_token indirection), block keys from this step's k/v.  Device time
    per launch with the L2 flushed before each; algorithmic bytes = q, out, block k/v, every context key and value
    and its slot id read once; FLOPs = 4 T H (ctx + 16) D per request."""
    from mfd_b200.ddtree_mode_attention import paged_mode_block_attention

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    Km, bsz = K_MODES, L_BLOCK
    T1 = Km * bsz
    ctxs = prefix_lengths(requests)
    g = torch.Generator(device=dev).manual_seed(11)
    slots = sum(ctxs) + 1024
    k_cache = (torch.randn(slots, HKV, D, generator=g, device=dev) * 0.5).bfloat16()
    v_cache = (torch.randn(slots, HKV, D, generator=g, device=dev) * 0.5).bfloat16()
    perm = torch.randperm(slots, generator=g, device=dev).to(torch.int32)
    r2t = torch.zeros(requests, max(ctxs) + 64, dtype=torch.int32, device=dev)
    off = 0
    for b, c in enumerate(ctxs):
        r2t[b, :c] = perm[off:off + c]
        off += c
    T = requests * T1
    q = torch.randn(T, H, D, generator=g, device=dev).bfloat16()
    k_new = (torch.randn(T, HKV, D, generator=g, device=dev) * 0.5).bfloat16()
    v_new = (torch.randn(T, HKV, D, generator=g, device=dev) * 0.5).bfloat16()
    rpi = torch.arange(requests, dtype=torch.int64, device=dev)
    ctx_t = torch.tensor(ctxs, dtype=torch.int64, device=dev)
    out = torch.empty_like(q)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    us = timed_us(lambda: paged_mode_block_attention(
        q=q, k_new=k_new, v_new=v_new, k_cache=k_cache, v_cache=v_cache, req_to_token=r2t, req_pool_indices=rpi,
        ctx_lens=ctx_t, num_modes=Km, block_size=bsz, scaling=D ** -0.5, num_ctx_splits=-1, out=out),
        steps, warmup, flush)
    alg = 2 * q.numel() * 2 + 2 * k_new.numel() * 2 + sum(2 * HKV * c * D * 2 for c in ctxs) + sum(ctxs) * 4
    flops = sum(4 * T1 * H * (c + bsz) * D for c in ctxs)
    pk = peaks()
    return {"kernel": "paged_mode_attn", "requests": requests,
            "workload": f"{requests} requests x {Km} modes x {bsz} queries x {H} heads, contexts U(1024, 8192) "
                        f"(mean {sum(ctxs) / len(ctxs):.0f}) in a paged cache of {slots} slots",
            "us_per_launch": round(us, 2), "algorithmic_bytes": alg, "flops": flops,
            "achieved_gbs": round(alg / us / 1e3, 1), "frac_of_hbm": round(alg / us / 1e3 / pk["hbm_gbs"], 4),
            "achieved_tflops": round(flops / us / 1e6, 1),
            "frac_of_tensor": round(flops / us / 1e6 / pk["bf16_tflops"], 4),
            "l2": "flushed (256 MB write) per launch"}


# ------------------------------------------------------------------------------------------------ CPU reference

def cpu_reference_inputs(req: int, prefix: int):
    """One request's host inputs for the reference's CPU path (generated outside any timed region)."""
    g = torch.Generator().manual_seed(1_000_003 * (req + 1))
    x = torch.randn(K_MODES, L_BLOCK, VOCAB, generator=g)
    ids = torch.randint(0, VOCAB, (K_MODES, L_BLOCK, 4), generator=g)
    x.scatter_add_(2, ids, torch.rand(K_MODES, L_BLOCK, 4, generator=g) * 6 + 4)
    q = torch.randn(1, H, W, D, generator=g).to(torch.bfloat16)
    kv = (torch.randn(2, 1, HKV, prefix + W, D, generator=g) * 0.5).to(torch.bfloat16)
    target = (torch.randn(1, W, VOCAB, generator=g) * 1.5).to(torch.bfloat16)
    return x, q, kv, target, prefix


def cpu_reference_request(inputs, temperature: float, ext) -> float:
    """The reference's CPU path for one request: float32 top-k + logsumexp (hf/ddtree.py:240-245), its C++ mixture
    builder (tree_build_ext.build_mixture), the compile_ddtree_tree mask + float32 SDPA with GQA repeat, the
    `sample` rule (argmax / softmax + multinomial, hf/model/utils.py:28-35) and its C++ walk.  Returns the seconds
    of that compute alone (inputs come from cpu_reference_inputs)."""
    x, q, kv, target, prefix = inputs
    t0 = time.perf_counter()
    top, tid = torch.topk(x, k=BUDGET, dim=-1)
    lz = torch.logsumexp(x, dim=-1, keepdim=True)
    lp = (top - lz).float()
    if ext is not None:
        tok, dep, parents, tree, vis = ext.build_mixture(lp.contiguous(), tid.contiguous(), torch.zeros(K_MODES), BUDGET)
    else:
        from oracle import oracle

        tok_np, dep_np, par_np = oracle.build_mixture(lp.numpy(), tid.numpy(), torch.zeros(K_MODES).numpy(), BUDGET)
        vis = torch.from_numpy(oracle.visibility(par_np))
        tree = None
    n = vis.shape[0]
    mask = torch.zeros(1, 1, n, prefix + n)
    blk = mask[0, 0, :, prefix:]
    blk.fill_(torch.finfo(torch.float32).min)
    blk.masked_fill_(vis, 0)
    G = H // HKV
    out = torch.nn.functional.scaled_dot_product_attention(
        q[:, :, :n].float(), kv[0].float().repeat_interleave(G, 1)[:, :, : prefix + n],
        kv[1].float().repeat_interleave(G, 1)[:, :, : prefix + n], attn_mask=mask, scale=D ** -0.5)
    logits = target[:, :n].float()
    if temperature < 1e-5:
        post = torch.argmax(logits, dim=-1)
    else:
        probs = torch.softmax(logits.view(-1, VOCAB) / temperature, dim=-1)
        post = torch.multinomial(probs, num_samples=1).view(1, n)
    if tree is not None:
        tree.follow(post[0].to(torch.long))
    del out
    return time.perf_counter() - t0


def reference_ext():
    try:
        from oracle import build_ref

        if build_ref.available():
            return build_ref.load("hf"), "reference"
    except Exception:
        pass
    return None, "port"


def cpu_reference_run(reqs, prefixes, temperature: float, ext, warmup: int = 1):
    """Compute seconds of the reference's CPU path per request over `reqs` (after `warmup` untimed requests); each
    request's inputs are generated before its timer starts."""
    for i in range(warmup):
        cpu_reference_request(cpu_reference_inputs(reqs[i % len(reqs)], prefixes[reqs[i % len(reqs)]]),
                              temperature, ext)
    secs = []
    for r in reqs:
        inputs = cpu_reference_inputs(r, prefixes[r])
        secs.append(cpu_reference_request(inputs, temperature, ext))
    return secs


def cpu_baseline(sample_requests: int = 3, temperature: float = 1.0):
    torch.set_num_threads(os.cpu_count() or 1)
    ext, kind = reference_ext()
    prefixes = prefix_lengths(TOTAL_REQUESTS)
    secs = cpu_reference_run(list(range(sample_requests)), prefixes, temperature, ext)
    per = statistics.mean(secs)
    return {"value": round(1.0 / per, 4), "unit": "trees/s", "cores": torch.get_num_threads(), "kind": kind,
            "sample": f"{sample_requests} requests of the benchmark workload (prefixes {prefixes[:sample_requests]}), "
                      f"compute only (inputs generated before each timer), mean {per * 1e3:.1f} ms per request, "
                      f"host {os.cpu_count()} cpus"}


# ------------------------------------------------------------------------------------------------ main

def timed_us(fn, steps: int, warmup: int, flush: torch.Tensor):
    """Mean device time of fn() in microseconds: warm-up, then each timed call after an L2 flush, bracketed by CUDA
    events on the current stream (a long device sleep first so host launch overhead is not measured)."""
    for _ in range(max(warmup, 3)):
        fn()
    times = []
    for _ in range(steps):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(2_000_000)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e) * 1e3)
    return statistics.mean(times)


def config_line(config: int, steps: int, warmup: int):
    """One BASELINE config's kernels alone (batch 1), against the roofline of that config's algorithmic work."""
    from mfd_b200 import ops

    dev = torch.device("cuda", 0)
    pk = peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    line = {"config": config, "peak_hbm_gbs": pk["hbm_gbs"], "peak_bf16_tflops": pk["bf16_tflops"],
            "peak_source": pk["source"]}
    if config in (0, 1):
        batch = Batch([0], [4096], dev, temperature=0.0, target_std=1.0, uniform_prefix=4096)
        step = Step(batch)
        step.run()
        if config == 0:
            def fn():
                ops.topk_logz(batch.draft.view(-1, VOCAB), BUDGET, ids_dtype=torch.int32,
                              out=(batch.top, batch.ids, batch.logz))
                ops.build_trees(batch.top.view(1, K_MODES, L_BLOCK, BUDGET), batch.ids.view(1, K_MODES, L_BLOCK, BUDGET),
                                None, BUDGET, tree=batch.tree, counts=batch.counts)
            nbytes, flops = K_MODES * L_BLOCK * VOCAB * 4, 0
            line["workload"] = "configs[0]: logits step + mixture tree, fp32 [8, 16, 151936], B=64"
        else:
            _, _, anc, _ = ops.build_trees(batch.top.view(1, K_MODES, L_BLOCK, BUDGET),
                                           batch.ids.view(1, K_MODES, L_BLOCK, BUDGET), None, BUDGET)
            def fn():
                ops.tree_attention(batch.q, batch.k, batch.v, anc, 4096, D ** -0.5, out=batch.attn_out)
            nbytes = (W * H * D * 2) * 2 + 2 * HKV * (4096 + W) * D * 2
            flops = 4 * W * H * (4096 + W) * D
            line["workload"] = "configs[1]: tree verify attention, 65 queries x 32 heads over 4096 + 65 keys (8 kv heads)"
    elif config == 2:
        import numpy as np
        import torch.nn.functional as F

        n, Hv, Hk = 64, 32, 16
        g = torch.Generator(device=dev).manual_seed(2)
        rng = np.random.default_rng(2)
        parents = [-1] + [int(rng.integers(0, i)) for i in range(1, n)]
        anc = torch.zeros(n, n, dtype=torch.int8)
        for i in range(n):
            if parents[i] >= 0:
                anc[i] = anc[parents[i]]
            anc[i, i] = 1
        anc = anc.to(dev)
        q = (F.normalize(torch.randn(n, Hk, D, generator=g, device=dev), dim=-1) * D ** -0.5).bfloat16()
        k = F.normalize(torch.randn(n, Hk, D, generator=g, device=dev), dim=-1).bfloat16()
        v = torch.randn(n, Hv, D, generator=g, device=dev).bfloat16()
        beta = torch.sigmoid(torch.randn(n, Hv, generator=g, device=dev))
        G = anc.float() @ (-F.softplus(torch.randn(n, Hv, generator=g, device=dev)))
        s0 = torch.randn(Hv, D, D, generator=g, device=dev) * 0.02
        u = torch.empty(n, Hv, D, device=dev)
        o = torch.empty_like(u)
        st = torch.empty(n, Hv, D, D, device=dev)
        uo_us = timed_us(lambda: ops.tree_gdn(q, k, v, G, beta, s0, anc, out=(u, o, None)), steps, warmup, flush)
        line["uo_us"] = round(uo_us, 2)
        line["uo_roofline_us"] = round((2 * n * Hk * D * 2 + n * Hv * D * 2 + Hv * D * D * 4 + 2 * n * Hv * D * 4)
                                       / (pk["hbm_gbs"] * 1e9) * 1e6, 2)
        # the layer's input preparation (causal conv of kernel 4 over each node's window -- its root path after
        # the conv state --, SiLU, l2 norms of q and k): tree_prep
        KC = 4
        cd = (2 * Hk + Hv) * D
        x = torch.randn(n, cd, generator=g, device=dev).bfloat16()
        conv_state = torch.randn(cd, KC, generator=g, device=dev).bfloat16()
        conv_w = (torch.randn(cd, KC, generator=g, device=dev) * 0.5).bfloat16()
        windows = []
        for i in range(n):
            path, j = [], i
            while j >= 0:
                path.append(KC + j)
                j = parents[j]
            windows.append((list(range(KC)) + path[::-1])[-KC:])
        conv_index = torch.tensor(windows, dtype=torch.int32, device=dev)
        prep_us = timed_us(lambda: ops.tree_prep(x, conv_state, conv_index, conv_w, Hk, Hv, D), steps, warmup, flush)
        prep_bytes = n * cd * 2 + 2 * cd * KC * 2 + n * KC * 4 + (2 * n * Hk * D + n * Hv * D) * 2
        line["prep_us"] = round(prep_us, 2)
        line["prep_roofline_us"] = round(prep_bytes / (pk["hbm_gbs"] * 1e9) * 1e6, 2)

        def fn():
            ops.tree_gdn(q, k, v, G, beta, s0, anc, emit_states=True, out=(u, o, st))
        nbytes = 2 * n * Hk * D * 2 + n * Hv * D * 2 + Hv * D * D * 4 + 2 * n * Hv * D * 4 + st.numel() * 4
        flops = 0
        line["workload"] = "configs[2]: tree GDN layer, 64 nodes, 32/16 heads d128, with per-node states"
    elif config == 3:
        from mfd_b200.mode_attention import mode_block_attention

        Km, bsz, ctx = 8, 16, 4096
        T = Km * bsz
        g = torch.Generator(device=dev).manual_seed(3)
        q = torch.randn(1, H, T, D, generator=g, device=dev).bfloat16()
        k = (torch.randn(1, HKV, ctx + T, D, generator=g, device=dev) * 0.5).bfloat16()
        v = (torch.randn(1, HKV, ctx + T, D, generator=g, device=dev) * 0.5).bfloat16()
        attn_us = timed_us(lambda: mode_block_attention(q, k, v, Km, bsz, D ** -0.5), steps, warmup, flush)
        attn_flops = 4 * T * H * (ctx + bsz) * D
        attn_bytes = 2 * (H * T * D * 2) + 2 * HKV * (ctx + T) * D * 2
        line["mode_attention_us"] = round(attn_us, 2)
        line["mode_attention_tensor_roofline_us"] = round(attn_flops / (pk["bf16_tflops"] * 1e12) * 1e6, 2)
        line["mode_attention_hbm_roofline_us"] = round(attn_bytes / (pk["hbm_gbs"] * 1e9) * 1e6, 2)
        # the mixture tree of sharp drafter logits, then greedy acceptance over target logits N(0,1) whose argmax
        # is forced along a seeded root-to-leaf path of depth 9
        batch = Batch([0], [64], dev, temperature=0.0, target_std=1.0, uniform_prefix=64)
        sharp_draft_logits(3, dev, batch.draft[0])
        step = Step(batch)
        step.run()
        t = batch.tree[0].cpu().tolist()
        path = forced_path(t[0], t[2], t[1], 9, seed=3)
        force_argmax(batch.target[0], t[0], path)
        o = ops.accept(batch.target, batch.tree[:, 0], batch.tree[:, 2], temperature=0.0, max_steps=L_BLOCK - 1,
                       out_len=L_BLOCK)
        line["tree_depth"] = max(t[1][: int(batch.counts[0]) + 1])
        line["forced_path_depth"] = len(path) - 1
        line["accept_len"] = int(o["accept_len"][0])
        line["accepted_tokens_match_path"] = o["accepted"][0, : len(path)].tolist() == path

        def fn():
            ops.accept(batch.target, batch.tree[:, 0], batch.tree[:, 2], temperature=0.0, max_steps=L_BLOCK - 1,
                       out_len=L_BLOCK)
        nbytes, flops = W * VOCAB * 2, 0
        line["workload"] = ("configs[3]: mode attention (128 queries x 32 heads over 4096 context + own 16-key block), "
                            "then a B=64 mixture tree of sharp drafter logits and greedy acceptance over target "
                            "logits bf16 [65, 151936] N(0,1) with the argmax forced along a depth-9 path; 'us' is "
                            "the acceptance")
    else:
        raise SystemExit(f"--config {config}: not available")
    us = timed_us(fn, steps, warmup, flush)
    line["us"] = round(us, 2)
    line["algorithmic_bytes"] = nbytes
    line["hbm_roofline_us"] = round(nbytes / (pk["hbm_gbs"] * 1e9) * 1e6, 2)
    line["frac_of_hbm_roofline"] = round(line["hbm_roofline_us"] / us, 4)
    if flops:
        line["flops"] = flops
        line["tensor_roofline_us"] = round(flops / (pk["bf16_tflops"] * 1e12) * 1e6, 2)
        line["frac_of_tensor_roofline"] = round(line["tensor_roofline_us"] / us, 4)
    line["l2"] = "flushed (256 MB write) before every timed call"
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mfd", choices=["mfd", "reference"])
    ap.add_argument("--requests", type=int, default=TOTAL_REQUESTS,
                    help="requests of the whole job (split over the GPUs: strong scaling)")
    ap.add_argument("--requests-per-gpu", type=int, default=REQUESTS_PER_GPU, help="--kernel lines only")
    ap.add_argument("--config", type=int, default=None, help="time one BASELINE config's kernels alone (1 GPU)")
    ap.add_argument("--no-extras", action="store_true", help="skip north_star / e2e / cpu_baseline")
    ap.add_argument("--north-star", action="store_true", help="time only the north-star step (1 GPU)")
    ap.add_argument("--kernel", default=None,
                    choices=["logits_step", "tree_build", "attention", "accept", "commit_kv", "gdn_commit",
                             "paged_mode_attn"],
                    help="time one kernel of the batch step alone (1 GPU)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        torch.set_num_threads(os.cpu_count() or 1)
        ext, kind = reference_ext()
        prefixes = prefix_lengths(args.requests)
        # one request of the workload per step, in request-id order; each request's inputs are generated before
        # its timer starts, so the sum below is the reference's compute alone
        reqs = [i % args.requests for i in range(args.steps)]
        secs = sum(cpu_reference_run(reqs, prefixes, 1.0, ext, warmup=args.warmup)) / args.steps
        value = 1.0 / secs
        line = {"impl": "reference", "metric": "verify-step trees/s (tree build + tree verify attention + accept)",
                "value": round(value, 4), "unit": "trees/s", "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(secs * 1e3, 2), "higher_is_better": True,
                "scaling": "none: one host process with all its cores, whatever the GPU count",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": f"configs[4] batched verify step ({args.requests} requests), one request per "
                                       "step on the host CPU, compute only",
                           "requests": args.requests, "budget": BUDGET, "modes": K_MODES, "block": L_BLOCK,
                           "vocab": VOCAB},
                "cpu_baseline": {"value": round(value, 4), "unit": "trees/s", "cores": torch.get_num_threads(),
                                 "kind": kind, "sample": f"{args.steps} requests of the workload (ids 0..), one per "
                                                         "step, inputs generated outside the timed compute"},
                "e2e": {"value": round(value, 4), "unit": "trees/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    if args.kernel == "paged_mode_attn":
        print(json.dumps(paged_line(args.steps, args.warmup, args.requests_per_gpu)))
        return
    if args.kernel is not None:
        fn = commit_line if args.kernel in ("commit_kv", "gdn_commit") else kernel_line
        print(json.dumps(fn(args.kernel, args.steps, args.warmup, args.requests_per_gpu)))
        return

    if args.north_star:
        torch.cuda.set_device(0)
        print(json.dumps(north_star(torch.device("cuda", 0), args.steps, args.warmup)))
        return
    if args.config is not None:
        torch.cuda.set_device(0)
        print(json.dumps(config_line(args.config, max(args.steps, 10), args.warmup)))
        return

    ws, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local if ws > 1 else 0)
    from mfd_b200 import _lib

    _lib.load()
    total = args.requests
    prefixes = prefix_lengths(total)
    reqs = partition(total, ws, rank, prefixes)
    batch = Batch(reqs, prefixes, dev)
    step = Step(batch)
    torch.cuda.synchronize()
    total_ms, per_kernel, clocks = time_steps(step, args.steps, args.warmup, ws, dev.index or 0)
    total_ms = max_over_ranks(ws, total_ms)
    ms_per_step = total_ms / args.steps
    value = total / (ms_per_step / 1e3)

    pk = peaks()
    # roofline of the dominant kernel: the logits step reads each request's float32 [8, 16, V] logits once
    rows = len(reqs) * K_MODES * L_BLOCK
    logits_bytes = rows * VOCAB * 4
    achieved = logits_bytes / (per_kernel["logits_step"] * 1e-6) / 1e9
    # roofline of the whole step: every input read once and every output written once, on the slowest rank
    step_bytes = batch.step_bytes()
    roof_ms = max_over_ranks(ws, step_bytes / (pk["hbm_gbs"] * 1e9) * 1e3)
    job_bytes = sum_over_ranks(ws, step_bytes)
    line = {
        "metric": "verify-step trees/s (tree build + tree verify attention + accept)",
        "value": round(value, 3), "unit": "trees/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"configs[4]: batched verify step, {total} requests partitioned over {ws} GPU(s), T=1",
                   "requests": total, "requests_per_gpu": len(reqs), "budget": BUDGET, "modes": K_MODES,
                   "block": L_BLOCK, "vocab": VOCAB, "heads": H, "kv_heads": HKV, "head_dim": D,
                   "prefix": "U(1024, 8192)", "l2": "inputs (~117 MB per request) far larger than L2",
                   "dtypes": "fp32 drafter logits, bf16 q/k/v and target logits, fp32 accumulation",
                   "parallelism": f"requests partitioned over {ws} GPU(s) (sorted by prefix, dealt round-robin), "
                                  "no collective"},
        "kernels_us_per_step": {k: round(v, 2) for k, v in per_kernel.items()},
        "roofline": {"kernel": "mfd_topk_logz (logits step)", "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                     "peak_source": pk["source"], "traffic": round(TOPK_TRAFFIC_PER_ROW * rows),
                     "traffic_source": "ncu capture of 1024 rows, scaled by rows",
                     "algorithmic_bytes_per_launch": logits_bytes},
        "step_roofline": {"bound": "hbm", "algorithmic_bytes_per_step": job_bytes,
                          "algorithmic_bytes_per_gpu": step_bytes, "roofline_ms": round(roof_ms, 4),
                          "achieved_gbs_per_gpu": round(step_bytes / (ms_per_step * 1e-3) / 1e9, 1),
                          "peak": pk["hbm_gbs"], "frac": round(roof_ms / ms_per_step, 4),
                          "what": "every input of the step read once (drafter logits, q, prefix + tree K/V, target "
                                  "logits, uniforms) and every output written once, on the slowest GPU"},
        "clocks": clocks,
        "gpu_launches": Step.LAUNCHES * args.steps,
    }
    if not args.no_extras:
        if rank == 0:
            line["north_star"] = north_star(dev, steps=20, warmup=args.warmup, graph=ws == 1)
        barrier(ws)
        line["e2e"] = e2e(dev, reqs, prefixes, steps=3, ws=ws)
        if ws == 1:
            line["cpu_baseline"] = cpu_baseline()
    if ws > 1:
        torch.distributed.barrier()
    if rank == 0:
        print(json.dumps(line))
    if ws > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
