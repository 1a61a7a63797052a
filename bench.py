#!/usr/bin/env python
"""Benchmark: positions evaluated per second on the grouped-decode wave.

Headline workload (one step = one wave): a bf16 HSTU chess model, d_model
512, 8 layers, 8 heads (head dims 64/64), random-initialised with the
reference's initialisers; 256 parent positions reached by seeded uniformly
random legal play of U[20, 200] plies from the start position (parent i uses
seed 1234 + i), each expanding ALL its legal moves (K = the parent's legal
move count) as depth-0 sibling rows that share the parent's game prefix in
the paged KV pool (16-token pages); every sibling carries its own UCI-sorted
legal move ids.  A step computes every sibling's policy logits at its legal
ids, their log-softmax, the WDL value and v = p(win) - p(loss), and appends
the sibling's KV to its turn arena.  Move generation and the board-state
encoding come from the worker-side chess module; no dataset or checkpoint
is available, so weights are random and positions are synthetic play.

--workload selects other measured workloads (d1024: the same wave shape on
the d1024/16L/16H model with long synthetic prefixes; halving: sequential-
halving search rounds with suffix chains; prefill_decode: jagged prefill and
one-token decode + KV-append steps).  The halving rounds (1,024 games per GPU,
rounds 32/16/8/4/2) are also measured in every default run and reported under
the "halving" key of the same line.

Reported:
  value  - positions/s with the wave's inputs resident in HBM (device time,
           CUDA events on the launching stream, max over ranks): the median
           of --passes timed passes of exactly --steps steps each.
  e2e    - positions/s through the C-ABI step with host buffers: pinned
           host->device copy of the packed wave, the step, device->host copy
           of its results (v and the legal log-softmax), synchronised every
           step; its p50 per-wave latency.
  service_api - the reference-compatible ActorInferenceServer.service() on
           the same wave (Python wire objects in and out), p50 latency.
  roofline - the dominant kernel's algorithmic work per launch over its
           average launch duration, against the measured peaks.  Launch
           durations come from CUDA events around each phase, recorded in a
           separate pass of the same steps right after the timed region (the
           events themselves add device time, so the headline value is timed
           without them).
  cpu_baseline - the reference's own decode path (its ActorInferenceServer,
           fp32 eager torch on the host cores, installed unmodified in
           baseline/_ref) on a bounded sample of the same workload.

--impl reference runs that reference path alone (the reference arm), and
adds the reference on this GPU under its CUDA bf16 autocast as a separate
field for comparison.

Multi-GPU (torchrun): each rank runs the same-size workload on its own games
(weak scaling, no collective on the data path).
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
if int(os.environ.get("WORLD_SIZE", "1")) > 1:
    # NCCL reads these when torch first loads it: its communicator init lines
    # (rank, device, ring) go to the run's log, whatever level the
    # environment had.  Stdout carries only rank 0's JSON line: file
    # descriptor 1 (NCCL's log included) is pointed at stderr, and the JSON
    # line goes to a copy of the original stdout.
    os.environ["NCCL_DEBUG"] = "INFO"
    os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(sys.stdout.fileno()), "w") if int(os.environ.get("RANK", "0")) == 0 else None
    os.dup2(sys.stderr.fileno(), sys.stdout.fileno())
else:
    _JSON_OUT = None


def emit(line: dict) -> None:
    """Print one result line (the JSON line of the run) on stdout."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()

METRIC = "positions evaluated/sec (grouped decode)"
# Per-workload defaults (per GPU; weak scaling under torchrun).
WORKLOADS = {
    "grouped": {"parents": 256, "plies": (20, 200), "siblings": None, "rounds": None},
    "d1024": {"parents": 512, "plies": (300, 600), "siblings": (40, 40), "rounds": None},
    "halving": {"parents": 1024, "plies": (40, 250), "siblings": None, "rounds": (32, 16, 8, 4, 2)},
    # games, plies log-uniform in [lo, hi], decode steps built (cycled when more are timed)
    "prefill_decode": {"parents": 1024, "plies": (1, 300), "siblings": None, "rounds": (50,)},
    # the headline wave through the dense model API and through the paged executors
    "model_api": {"parents": 256, "plies": (20, 200), "siblings": None, "rounds": None},
}
UNIT = "positions/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
REF_PATH = os.path.join(ROOT, "baseline", "_ref")


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--passes", type=int, default=3, help="timed passes of --steps steps; the median is reported")
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", choices=list(WORKLOADS), default="grouped")
    ap.add_argument("--parents", type=int, default=None)
    ap.add_argument("--plies", type=int, nargs=2, default=None)
    ap.add_argument("--siblings", type=int, nargs=2, default=None)
    ap.add_argument("--rounds", type=int, nargs="+", default=None, help="halving: arms per round")
    ap.add_argument("--no-halving", action="store_true", help="skip the extra halving-rounds measurement")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-service", action="store_true")
    ap.add_argument("--no-reference-cuda", action="store_true", help="reference arm: skip its CUDA bf16 run")
    ap.add_argument("--cpu-sample-parents", type=int, default=4)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args(argv)
    for k, v in WORKLOADS[args.workload].items():
        if getattr(args, k) is None:
            setattr(args, k, v)
    return args


def workload_args(args, name):
    """A copy of ``args`` for workload ``name`` with that workload's defaults."""
    sub = argparse.Namespace(**vars(args))
    sub.workload = name
    for k, v in WORKLOADS[name].items():
        setattr(sub, k, v)
    return sub


def dist_env():
    from imba_chess_b200.shard import dist_env as env

    return env()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {k: float(p[k]) for k in PEAKS_FALLBACK}, "measured"
    except Exception:
        return dict(PEAKS_FALLBACK), "fallback"


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


# ----------------------------------------------------------------------
# Workload
# ----------------------------------------------------------------------
def workload(args, rank, world=1):
    """This rank's parents: global parent i (seed 1234 + i) belongs to rank
    i % world (imba_chess_b200.shard.shard_games); every rank gets
    ``--parents`` of them (weak scaling)."""
    from imba_chess_b200 import synth
    from imba_chess_b200.shard import shard_games

    mine = shard_games(args.parents * world, rank, world)
    if args.workload in ("grouped", "model_api"):
        dims = synth.D512
        parts = [synth.chess_grouped_wave(n_parents=1, plies=tuple(args.plies), seed=1234 + i) for i in mine]
    else:
        dims = synth.D1024
        parts = [synth.grouped_wave(dims, n_parents=1, plies=tuple(args.plies), siblings=tuple(args.siblings),
                                    seed=1234 + i) for i in mine]
    wave = synth.GroupedWave(
        prefix_tokens=[p.prefix_tokens[0] for p in parts],
        row_tokens=synth.concat_tokens([p.row_tokens for p in parts]),
        group_index=np.concatenate([np.full(p.num_rows, g, dtype=np.int64) for g, p in enumerate(parts)]),
        legal_ids=[ids for p in parts for ids in p.legal_ids],
    )
    return dims, wave


def workload_config(args):
    if args.workload == "prefill_decode":
        return {
            "workload": "jagged prefill + incremental decode: bf16 HSTU d512/8L/8H (max_pos 1024), "
                        f"{args.parents} games, prefixes log-uniform in [{args.plies[0]},{args.plies[1]}] plies "
                        "prefilled in packed batches of <= 32,768 tokens, then one-token decode + KV append "
                        "steps of every game with its legal log-softmax and v (one step = one token per game)",
            "games_per_gpu": args.parents,
            "page_tokens": 16,
            "l2": "inputs larger than L2 (prefix KV read per step > 126 MB at full size)",
        }
    if args.workload == "halving":
        return {
            "workload": "sequential-halving search rounds: bf16 HSTU d512/8L/8H (max_pos 513), "
                        f"{args.parents} games, prefixes U[{args.plies[0]},{args.plies[1]}] plies, rounds of "
                        f"{'/'.join(str(k) for k in args.rounds)} surviving arms per game, round r evaluates one "
                        "node per arm at depth r whose suffix is the arm's chain in the turn arena; "
                        "one step = every round of every game",
            "games_per_gpu": args.parents,
            "page_tokens": 16,
            "l2": "inputs larger than L2 (prefix KV read per round > 126 MB at full size)",
        }
    if args.workload == "model_api":
        return {
            "workload": "grouped-decode wave through the reference-compatible APIs: bf16 HSTU d512/8L/8H "
                        f"(max_pos 513), {args.parents} parents from random legal play of "
                        f"U[{args.plies[0]},{args.plies[1]}] plies, every legal move as a depth-0 sibling; "
                        "value: B200HSTUChessModel.forward_decode_grouped on the reference's padded [G,H,maxP,d] "
                        "prefix stack (device tensors, full 1,970-way logits and new per-layer KV returned, "
                        "synchronised per call); paged: the rollout executor on pool-resident prefixes",
            "parents_per_gpu": args.parents,
            "page_tokens": 16,
            "l2": "inputs larger than L2 (prefix stack per call > 126 MB)",
        }
    if args.workload == "d1024":
        return {
            "workload": "grouped-decode wave: bf16 HSTU d1024/16L/16H (max_pos 1024), head dims 64/64, "
                        f"{args.parents} parents, synthetic prefixes U[{args.plies[0]},{args.plies[1]}] plies, "
                        f"U[{args.siblings[0]},{args.siblings[1]}] depth-0 siblings each, 16-token KV pages",
            "parents_per_gpu": args.parents,
            "page_tokens": 16,
            "l2": "inputs larger than L2 (prefix KV read per step > 126 MB at full size)",
        }
    return {
        "workload": "grouped-decode wave: bf16 HSTU d512/8L/8H (max_pos 513), head dims 64/64, "
                    f"{args.parents} parents from random legal play of U[{args.plies[0]},{args.plies[1]}] plies, "
                    "every legal move of each parent as a depth-0 sibling (K = its legal move count), "
                    "16-token KV pages",
        "parents_per_gpu": args.parents,
        "page_tokens": 16,
        "l2": "inputs larger than L2 (prefix KV read per step > 126 MB at full size)",
    }


def full_config(args, rows_all, world):
    return workload_config(args) | {"rows_per_step": int(rows_all), "parallelism": f"dp{world} (independent games)"}


# ----------------------------------------------------------------------
# Clock sampling during the timed region
# ----------------------------------------------------------------------
REASON_FIELDS = (
    ("hw_slowdown", "clocks_event_reasons.hw_slowdown"),
    ("hw_thermal_slowdown", "clocks_event_reasons.hw_thermal_slowdown"),
    ("sw_thermal_slowdown", "clocks_event_reasons.sw_thermal_slowdown"),
    ("sw_power_cap", "clocks_event_reasons.sw_power_cap"),
)


class ClockSampler:
    def __init__(self, device_index: int) -> None:
        self.samples: list[tuple[float, float, list[str]]] = []
        self._proc = None
        self._thread = None
        q = ",".join(["clocks.sm", "clocks.max.sm"] + [f for _, f in REASON_FIELDS])
        ident = str(device_index)
        try:
            import torch

            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            pass
        self._cmd = ["nvidia-smi", "-i", ident, f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "200"]

    def start(self):
        try:
            self._proc = subprocess.Popen(self._cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self._proc = None
            return
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()

    def _read(self):
        for line in self._proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 2 + len(REASON_FIELDS):
                continue
            try:
                sm, mx = float(parts[0]), float(parts[1])
            except ValueError:
                continue
            active = [name for (name, _), v in zip(REASON_FIELDS, parts[2:]) if v.lower() == "active"]
            self.samples.append((sm, mx, active))

    def stop(self):
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except Exception:
                self._proc.kill()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s in self.samples if s[0] > 0.5 * s[1]] or self.samples
        reasons = sorted({r for s in loaded for r in s[2]})
        return {
            "sm_mhz": statistics.median(s[0] for s in loaded),
            "sm_max_mhz": max(s[1] for s in self.samples),
            "reasons": reasons,
            "samples": len(self.samples),
        }


# ----------------------------------------------------------------------
# The reference's own decode path (baseline/_ref), CPU fp32 and CUDA bf16
# ----------------------------------------------------------------------
SIDE_KEYS = ("turn_id", "castle_id", "ep_file_id", "halfmove_bucket_id", "fullmove_bucket_id")


class ReferenceServerRun:
    """The reference's ``ActorInferenceServer`` (installed unmodified under
    baseline/_ref, imported through the oracle's import shims) serving the
    roots and the wave of the given parents, through the reference's own torch
    decode path (actor_server.py:519-551 -> forward_decode_grouped,
    hstu_model.py:651-752).  CPU: fp32 eager on all host threads; CUDA: the
    server's own bf16 autocast (position_evaluator.py:184-194)."""

    def __init__(self, dims, wave, parents, device: str, dtype_name: str, root_chunk: int = 8):
        from oracle import ref_shims

        ref_shims.install(REF_PATH)
        import torch
        from imba_chess.config import ModelConfig
        from imba_chess.eval.actor_protocol import RootEvalRequest, WaveRequest, WaveRow
        from imba_chess.eval.actor_server import ActorInferenceServer
        from imba_chess.model import HSTUChessModel, build_hstu_chess_config

        from imba_chess_b200 import synth

        self.torch = torch
        self.device = torch.device(device)
        if self.device.type == "cpu":
            torch.set_num_threads(os.cpu_count() or 1)
        cfg = build_hstu_chess_config(
            ModelConfig(model_dim=dims.model_dim, linear_hidden_dim=dims.linear_dim,
                        attention_dim=dims.attention_dim, num_heads=dims.num_heads, num_layers=dims.num_layers,
                        dropout=0.0, max_position_embeddings=dims.max_pos, halfmove_vocab_size=dims.halfmove_vocab,
                        fullmove_vocab_size=dims.fullmove_vocab, enable_value_head=dims.value_head),
            move_vocab_size=dims.vocab)
        model = HSTUChessModel(cfg).eval()
        sd = synth.make_state_dict(dims, 2, profile="reference")
        model.load_state_dict({k: torch.from_numpy(v.copy()) for k, v in sd.items()}, strict=True)
        model = model.to(self.device)
        dtype = torch.bfloat16 if dtype_name == "bf16" else torch.float32
        self.server = ActorInferenceServer(model=model, device=self.device, dtype=dtype)
        # roots in chunks (the reference merges one service() call's roots into one jagged prefill)
        for c in range(0, len(parents), root_chunk):
            roots = [RootEvalRequest(worker_id=g, turn_id=0, legal_vocab_ids=[2],
                                     batch_arrays=synth.root_batch_arrays(wave.prefix_tokens[g]))
                     for g in parents[c:c + root_chunk]]
            self.server.service(roots)
        rt = wave.row_tokens
        self.requests = []
        self.rows = 0
        for g in parents:
            rows = []
            for i in np.nonzero(wave.group_index == g)[0]:
                bs = {"piece_ids": rt["piece_ids"][i].tolist(), **{k: int(rt[k][i]) for k in SIDE_KEYS}}
                rows.append(WaveRow(node_id=int(i), parent_id=None, prev_move_vocab_id=int(rt["prev_move_id"][i]),
                                    board_state=bs, legal_vocab_ids=[int(x) for x in wave.legal_ids[i]]))
            if rows:
                self.requests.append(WaveRequest(worker_id=g, turn_id=0, rows=rows))
                self.rows += len(rows)

    def step(self) -> float:
        """One wave through service() (inputs from Python objects, outputs
        back as Python floats); returns its wall time in seconds."""
        t0 = time.perf_counter()
        self.server.service(self.requests)
        return time.perf_counter() - t0


def sample_parents(wave, n):
    """The wave's first ``n`` parents that have sibling rows."""
    counts = np.bincount(wave.group_index, minlength=len(wave.prefix_tokens))
    return [int(g) for g in np.nonzero(counts)[0][:n]]


def reference_cpu_rate(dims, wave, n_parents, steps=None, seconds=None, warmup=1):
    """(rows, per-step seconds) of the reference's CPU path on the wave's
    first ``n_parents`` parents with rows."""
    run = ReferenceServerRun(dims, wave, sample_parents(wave, n_parents), "cpu", "f32")
    for _ in range(max(warmup, 1)):
        run.step()
    times = []
    t_start = time.perf_counter()
    while True:
        times.append(run.step())
        if steps is not None and len(times) >= steps:
            break
        if steps is None and time.perf_counter() - t_start >= seconds:
            break
    return run.rows, times


def reference_cuda_rate(dims, wave, steps, warmup=1):
    """(rows, per-step seconds) of the reference on this GPU (bf16 autocast)
    over the full wave."""
    run = ReferenceServerRun(dims, wave, list(range(len(wave.prefix_tokens))), "cuda:0", "bf16")
    for _ in range(max(warmup, 1)):
        run.step()
    return run.rows, [run.step() for _ in range(steps)]


def cpu_oracle_rate(dims, wave, n_sample_parents, steps):
    """Rows/s of the numpy oracle port's grouped decode (legal log-priors and
    v included) on the first ``n_sample_parents`` parents of the wave."""
    from imba_chess_b200 import synth
    from oracle.hstu_np import OracleModel, gather_legal, log_softmax_f32, value_stm

    sd = synth.make_state_dict(dims, 2, profile="reference")
    orc = OracleModel(sd, dims)
    gsel = sample_parents(wave, n_sample_parents)
    lens = [wave.prefix_lens[g] for g in gsel]
    pref = [orc.forward(wave.prefix_tokens[g], [0, lens[i]])["kv_caches"] for i, g in enumerate(gsel)]
    max_p = max(lens)
    grouped = []
    for l in range(dims.num_layers):
        ks = np.stack([np.pad(p[l][0], ((0, 0), (0, max_p - p[l][0].shape[1]), (0, 0))) for p in pref])
        vs = np.stack([np.pad(p[l][1], ((0, 0), (0, max_p - p[l][1].shape[1]), (0, 0))) for p in pref])
        grouped.append((ks, vs))
    rows = np.nonzero(np.isin(wave.group_index, gsel))[0]
    tok = synth.slice_tokens(wave.row_tokens, rows)
    gi = np.searchsorted(np.asarray(gsel), wave.group_index[rows])  # group index within the sample
    legal = [wave.legal_ids[i] for i in rows]
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        out = orc.forward_decode_grouped(new_token_batch=tok, positions=np.asarray(lens)[gi], group_index=gi,
                                         prefix_kv_grouped=grouped, prefix_lens_list=lens)
        for x in gather_legal(out["logits"], legal):
            log_softmax_f32(x)
        value_stm(out["value_logits"])
        times.append(time.perf_counter() - t0)
    return len(rows), times


def _torch_version():
    import torch

    return torch.__version__


def run_reference(args):
    """Reference arm: the reference's own decode path (its ActorInferenceServer
    on the host cores, fp32 eager, all host threads), each step a bounded
    sample (the wave's first --cpu-sample-parents parents); rank 0 only."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    if args.workload not in ("grouped", "d1024"):
        emit({"impl": "reference", "unavailable": "the reference arm is timed on the grouped-decode wave workloads "
                                                  "only"})
        return
    if not os.path.isdir(os.path.join(REF_PATH, "imba_chess")):
        emit({"impl": "reference", "unavailable": "the reference is not installed under baseline/_ref"})
        return
    dims, wave = workload(args, 0, world)
    rows_all = wave.num_rows * world
    n_rows, times = reference_cpu_rate(dims, wave, args.cpu_sample_parents, steps=args.steps, warmup=args.warmup)
    total = float(sum(times))
    value = n_rows * len(times) / total
    cores = os.cpu_count() or 1
    sample = (f"the wave's first {args.cpu_sample_parents} parents with rows ({n_rows} sibling rows) of "
              f"{args.parents} per step, reference ActorInferenceServer.service(), fp32 eager torch")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * total / len(times),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": full_config(args, rows_all, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "reference", "sample": sample,
                         "cpu_model": cpu_model(), "torch": _torch_version()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    import torch

    if not args.no_reference_cuda and torch.cuda.is_available():
        # For comparison only (not the arm): the reference on this GPU under its
        # CUDA bf16 autocast, full wave per step.
        csteps = max(1, min(args.steps, 5))
        rows, ct = reference_cuda_rate(dims, wave, csteps, warmup=1)
        line["reference_cuda_bf16"] = {
            "value": rows * len(ct) / sum(ct), "unit": UNIT, "ms_per_step": 1000.0 * sum(ct) / len(ct),
            "rows_per_step": rows, "steps": csteps,
            "what": "reference ActorInferenceServer.service() on cuda:0 with bf16 autocast, eager torch, full wave"}
    emit(line)


# ----------------------------------------------------------------------
# B200 arm
# ----------------------------------------------------------------------
def prefill(model, pool, seqs, tokens, device, max_tokens=32768):
    """Prefill sequences in packed batches of at most max_tokens tokens (setup, untimed)."""
    import torch

    from imba_chess_b200.plan import DeviceStep
    from imba_chess_b200.steps import root_plan

    i = 0
    while i < len(seqs):
        j, n = i, 0
        while j < len(seqs) and (j == i or n + int(tokens[j]["piece_ids"].shape[0]) <= max_tokens):
            n += int(tokens[j]["piece_ids"].shape[0])
            j += 1
        plan, _ = root_plan(seqs[i:j], tokens[i:j])
        model.run(DeviceStep(plan, device), pool)
        i = j
    torch.cuda.synchronize()
    model.check_status()


def build_waves(args, dims, model, device, rank, world):
    """The plans of one timed step and the pool they run on.  grouped / d1024:
    one wave of every parent's depth-0 siblings; halving: one wave per round,
    round r evaluating one node per surviving arm at depth r (its parent chain
    from the earlier rounds as suffix keys)."""
    from imba_chess_b200 import synth
    from imba_chess_b200.kvpool import KVSequence
    from imba_chess_b200.plan import piece_ids_from_tokens, side_ids_from_tokens
    from imba_chess_b200.shard import shard_games
    from imba_chess_b200.steps import WaveGroup, root_plan, wave_plan

    if args.workload == "prefill_decode":
        mine = shard_games(args.parents * world, rank, world)
        rngs = [np.random.default_rng(1234 + i) for i in mine]
        lo, hi = np.log(args.plies[0]), np.log(args.plies[1])
        plies = [int(np.exp(r.uniform(lo, hi))) for r in rngs]
        prefixes = [synth.game_tokens(r, n, dims) for r, n in zip(rngs, plies)]
        lens = [int(p["piece_ids"].shape[0]) for p in prefixes]
        steps = args.rounds[0]
        G = len(mine)
        pool = model.new_pool(sum(-(-(n + steps) // 16) for n in lens) + G + 64)
        seqs = [KVSequence(pool) for _ in lens]
        prefill_plans = []
        i = 0
        while i < G:  # packed batches of <= 32,768 tokens
            j, n = i, 0
            while j < G and (j == i or n + lens[j] <= 32768):
                n += lens[j]
                j += 1
            prefill_plans.append(root_plan(seqs[i:j], prefixes[i:j])[0])
            i = j
        plans = []
        for _ in range(steps):
            tok = [synth.random_tokens(r, 1, dims) for r in rngs]
            legal = [synth.random_legal_ids(r, int(r.integers(20, 41)), dims.vocab) for r in rngs]
            plans.append(root_plan(seqs, tok, legal_last=legal)[0])
        return pool, plans, prefill_plans
    if args.workload != "halving":
        _, wave = workload(args, rank, world)
        lens = wave.prefix_lens
        B = wave.num_rows
        pool = model.new_pool(sum(-(-n // 16) for n in lens) + 4 * (-(-B // 16)) + 2 * len(lens) + 64)
        seqs = [KVSequence(pool) for _ in lens]
        prefill(model, pool, seqs, wave.prefix_tokens, device)
        order = np.argsort(wave.group_index, kind="stable")
        arenas = [KVSequence(pool) for _ in lens]
        counts = np.bincount(wave.group_index, minlength=len(lens))
        groups = [WaveGroup(prefix=seqs[g], prefix_len=lens[g], arena=arenas[g], chains=[[]] * int(counts[g]))
                  for g in range(len(lens))]
        tok = synth.slice_tokens(wave.row_tokens, order)
        plan, _ = wave_plan(groups, piece_ids_from_tokens(tok), side_ids_from_tokens(tok),
                            [wave.legal_ids[i] for i in order])
        return pool, [plan], wave
    mine = shard_games(args.parents * world, rank, world)
    rngs = [np.random.default_rng(1234 + i) for i in mine]
    prefixes = [synth.game_tokens(r, int(r.integers(args.plies[0], args.plies[1] + 1)), dims) for r in rngs]
    lens = [int(p["piece_ids"].shape[0]) for p in prefixes]
    G, per_game = len(mine), sum(args.rounds)
    pool = model.new_pool(sum(-(-n // 16) for n in lens) + G * (-(-per_game // 16) + 1) + 64)
    seqs = [KVSequence(pool) for _ in lens]
    prefill(model, pool, seqs, prefixes, device)
    arenas = [KVSequence(pool) for _ in lens]
    chains = [[[] for _ in range(args.rounds[0])] for _ in range(G)]
    plans = []
    for K in args.rounds:
        groups = [WaveGroup(prefix=seqs[g], prefix_len=lens[g], arena=arenas[g], chains=[chains[g][a] for a in range(K)])
                  for g in range(G)]
        tok = synth.concat_tokens([synth.random_tokens(r, K, dims) for r in rngs])
        legal = [synth.random_legal_ids(r, int(r.integers(20, 41)), dims.vocab) for r in rngs for _ in range(K)]
        plan, own = wave_plan(groups, piece_ids_from_tokens(tok), side_ids_from_tokens(tok), legal)
        for g in range(G):
            for a in range(K):
                chains[g][a] = chains[g][a] + [own[g][a]]
        plans.append(plan)
    return pool, plans, None


PHASES = ("embed", "ln", "uvqk_gemm", "attention", "gate", "out_gemm", "final_ln", "policy_gemm", "value_gemm",
          "value_legal")


def phase_times(events, L):
    """Per-phase durations (ms) of one profiled step from its events."""
    t = {p: 0.0 for p in PHASES}
    e = events
    t["embed"] += e[0].elapsed_time(e[1])
    for l in range(L):
        b = 1 + 5 * l
        t["ln"] += e[b].elapsed_time(e[b + 1])
        t["uvqk_gemm"] += e[b + 1].elapsed_time(e[b + 2])
        t["attention"] += e[b + 2].elapsed_time(e[b + 3])
        t["gate"] += e[b + 3].elapsed_time(e[b + 4])
        t["out_gemm"] += e[b + 4].elapsed_time(e[b + 5])
    b = 1 + 5 * L
    t["final_ln"] += e[b].elapsed_time(e[b + 1])
    t["policy_gemm"] += e[b + 1].elapsed_time(e[b + 2])
    t["value_gemm"] += e[b + 2].elapsed_time(e[b + 3])
    t["value_legal"] += e[b + 3].elapsed_time(e[b + 4])
    return t


def algorithmic_work(dims, plan, eb=2):
    """Per-launch algorithmic FLOPs (tensor-bound phases) or bytes (HBM-bound
    phases) of one wave step, and launches per step."""
    R = plan.num_rows
    d, L, H, dqk, dv, V = dims.model_dim, dims.num_layers, dims.num_heads, dims.attention_dim, dims.linear_dim, dims.vocab
    uvqk_n = 2 * H * (dqk + dv)
    board_mac = 2 * (64 * 64 * 192 + 2 * 4 * 64 * 64 * 16 + 64 * 64 * 64 + 2 * 64 * 64 * 128) + 64 * d
    prefix_tokens = int(plan.row_vis[np.unique(plan.row_group, return_index=True)[1]].sum()) if R else 0
    kv_tok = H * (dqk + dv) * eb
    extras = int(plan.extra_slot.shape[0])
    nl = 0 if plan.legal_ids is None else int(plan.legal_ids.shape[0])
    # bf16 path: the attention kernel also applies the output norm and the u
    # gate (reads q, u; writes gated bf16), and without a full-logits request
    # the legal logits are fp32 gathers in the value / legal pass (policy rows
    # of the legal ids, mostly served from L2), so those two phases launch
    # nothing of their own.
    # With more than 8 heads a CTA holds half of them: attention writes fp32
    # and the norm / gate is its own pass.
    fused = H <= 8
    attn_out = R * H * dv * (eb + eb) if fused else R * H * dv * 4
    attn_bytes = prefix_tokens * kv_tok + extras * kv_tok + R * H * dqk * eb + attn_out
    work = {
        "embed": ("tensor", 2.0 * board_mac * R, 1),
        "ln": ("hbm", R * d * (4 + eb), L),
        "uvqk_gemm": ("tensor", 2.0 * R * d * uvqk_n, L),
        "attention": ("hbm", attn_bytes, L),
        "gate": ("hbm", R * H * dv * (4 + eb + eb), L),
        "out_gemm": ("tensor", 2.0 * R * H * dv * d, L),
        "final_ln": ("hbm", R * d * (4 + 4 + 2 * eb), 1),
        "value_gemm": ("tensor", 2.0 * R * d * (d // 2), 1),
        "value_legal": ("hbm", R * (d // 2) * 4 + nl * (d * 4 + 12) + R * (d * 4 + 16), 1),
    }
    if fused:
        del work["gate"]
    return work


def read_traffic():
    """Per-row DRAM traffic of each phase's kernel from the committed ncu
    summary (profiles/ncu_traffic_per_row.txt: '<phase> <bytes per row>')."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic_per_row.txt")
    out = {}
    if os.path.exists(path):
        for line in open(path):
            parts = line.split()
            if len(parts) == 2 and not line.startswith("#"):
                try:
                    out[parts[0]] = float(parts[1])
                except ValueError:
                    pass
    return out


def count_launches(dims, plan):
    """Kernel launches of one bf16 wave step (legal logits only): board
    encoder, content projection GEMM, L x (input LN, uvqk GEMM, attention with
    the fused norm / gate (a separate gate pass above 8 heads), output GEMM),
    final LN, value GEMM, value / legal."""
    return 2 + (4 if dims.num_heads <= 8 else 5) * dims.num_layers + 3


def measure(args, model, dims, device, rank, world, sampler=None):
    """Everything measured on one workload: the timed passes (device time,
    max over ranks), the per-phase profile pass, the roofline of the dominant
    kernel and the end-to-end pass through the C ABI with host buffers."""
    import ctypes

    import torch
    import torch.distributed as dist

    from imba_chess_b200 import _native
    from imba_chess_b200.plan import DeviceStep
    from imba_chess_b200.shard import reduce_max, reduce_sum

    pool, plans, extra = build_waves(args, dims, model, device, rank, world)
    stream = torch.cuda.current_stream(device)
    L = dims.num_layers
    n_ev = int(model._lib.imba_profile_event_count(model._handle))

    class Wave:
        def __init__(self, plan, outputs=True):
            self.plan = plan
            self.R = plan.num_rows
            self.NL = 0 if plan.legal_ids is None else int(plan.legal_ids.shape[0])
            self.outputs = outputs  # False: KV append only (a prefill batch)
            self.dstep = DeviceStep(plan, device, pinned=True)
            # The step's results: v and the masked policy log-softmax at the
            # legal ids (the workload's outputs), read back every e2e step.
            self.out = torch.empty(self.R + self.NL, dtype=torch.float32, device=device)
            self.v, self.lp = self.out[: self.R], self.out[self.R :]
            self.host_out = torch.empty(self.out.numel(), dtype=torch.float32, pin_memory=True)

        def run(self):
            if self.outputs:
                model.run(self.dstep, pool, value_stm=self.v, legal_logprob=self.lp)
            else:
                model.run(self.dstep, pool)

        def run_profiled(self, arr):
            desc = self.dstep.desc
            desc.value_stm = self.v.data_ptr() if self.outputs else None
            desc.legal_logits = None
            desc.legal_logprob = self.lp.data_ptr() if self.outputs and self.NL else None
            desc.logits = None
            desc.value_logits = None
            desc.hidden = None
            desc.status = model._status.data_ptr()
            ws = model.workspace(self.R)
            code = model._lib.imba_step_profiled(model._handle, ctypes.byref(desc), ctypes.byref(pool.desc),
                                                 ws.data_ptr(), ws.numel(), stream.cuda_stream, arr, n_ev)
            _native.check(code, "imba_step_profiled")

    def make_events():
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_ev)]
        for e in evs:
            e.record(stream)  # creates the handle
        arr = (ctypes.c_void_p * n_ev)(*[e.cuda_event for e in evs])
        return evs, arr

    waves = [Wave(p) for p in plans]
    cycle = args.workload == "prefill_decode"  # one prebuilt decode step per bench step

    def step_waves(i):
        return [waves[i % len(waves)]] if cycle else waves

    R = sum(w.R for w in step_waves(0))  # positions per step on this rank
    result = {}
    if args.workload == "prefill_decode":
        # The jagged prefill, timed apart (device time of its packed batches).
        # Re-running a prefill batch rewrites the same KV slots with the same
        # values, so it is warmed up once, timed, then run once more with
        # events between its phases.
        psteps = [Wave(p, outputs=False) for p in extra]
        for w in psteps:
            w.run()
        torch.cuda.synchronize()
        model.check_status()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for w in psteps:
            w.run()
        e1.record(stream)
        torch.cuda.synchronize()
        model.check_status()
        ntok = sum(p.num_rows for p in extra)
        pms = e0.elapsed_time(e1)
        p_ev = [make_events() for _ in psteps]
        torch.cuda.synchronize()
        for w, (_, arr) in zip(psteps, p_ev):
            w.run_profiled(arr)
        torch.cuda.synchronize()
        model.check_status()
        p_phase = {p: 0.0 for p in PHASES}
        for evs, _ in p_ev:
            for k, v in phase_times(evs, L).items():
                p_phase[k] += v
        # Its roofline: the tensor work of every token (board encoder, content,
        # trunk and value GEMMs) plus the causal attention products over each
        # token's visible keys, against the sustained bf16 peak.
        d, H = dims.model_dim, dims.num_heads
        qkv = dims.attention_dim + dims.linear_dim
        board_mac = 2 * (64 * 64 * 192 + 2 * 4 * 64 * 64 * 16 + 64 * 64 * 64 + 2 * 64 * 64 * 128) + 64 * d
        dense_mac = (board_mac + 3 * 64 * d + dims.num_layers * (d * 2 * H * qkv + H * dims.linear_dim * d)
                     + d * (d // 2))
        attn_mac = sum(int(p.row_vis.astype(np.int64).sum()) for p in extra) * dims.num_layers * H * qkv
        flop = 2.0 * (dense_mac * ntok + attn_mac)
        peaks, _src = load_peaks()
        achieved = flop / (pms / 1000.0) / 1e12
        result["prefill"] = {"tokens": int(ntok), "batches": len(extra), "ms": round(pms, 3),
                             "tokens_per_s": ntok / (pms / 1000.0),
                             "phases_ms": {k: round(v, 4) for k, v in p_phase.items() if v > 0},
                             "roofline": {"bound": "tensor", "achieved": round(achieved, 2),
                                          "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                                          "frac": round(achieved / peaks["bf16_tflops_sustained"], 4),
                                          "gflop": round(flop / 1e9, 1)}}

    def step_plain(i):
        for w in step_waves(i):
            w.run()

    for i in range(args.warmup):
        step_plain(i)
    torch.cuda.synchronize()
    model.check_status()
    if sampler is not None:
        sampler.start()
        time.sleep(0.3)
    pass_ms = []
    for _ in range(max(args.passes, 1)):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for i in range(args.steps):
            step_plain(i)
        t_end.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        pass_ms.append(reduce_max(t_start.elapsed_time(t_end), device))
    if sampler is not None:
        sampler.stop()
    model.check_status()
    # Per-phase breakdown: a separate pass of the same steps with CUDA events
    # between phases (the events add device time, so this pass is not the
    # headline number).
    ev_sets = [[make_events() for _ in step_waves(i)] for i in range(args.steps)]
    torch.cuda.synchronize()
    for i in range(args.steps):
        for w, (_, arr) in zip(step_waves(i), ev_sets[i]):
            w.run_profiled(arr)
    torch.cuda.synchronize()
    model.check_status()
    elapsed_ms = statistics.median(pass_ms)
    rows_all = reduce_sum(R, device)  # positions per step over all ranks
    ms_per_step = elapsed_ms / args.steps
    value = rows_all * args.steps / (elapsed_ms / 1000.0)

    # Per-phase device times (averaged over the timed steps, summed over the
    # step's waves) and the algorithmic work of a step.
    acc = {p: 0.0 for p in PHASES}
    for sets in ev_sets:
        for evs, _ in sets:
            for k, v in phase_times(evs, L).items():
                acc[k] += v
    per_step = {k: v / args.steps for k, v in acc.items()}
    work = {}
    for i in range(args.steps):
        for w in step_waves(i):
            for k, (bound, amount, launches) in algorithmic_work(dims, w.plan).items():
                b0, a0, l0 = work.get(k, (bound, 0.0, 0))
                work[k] = (bound, a0 + amount * launches, l0 + launches)
    # per-launch work: the timed steps' total work over their launches; launches per step
    work = {k: (bnd, total / n, n // args.steps) for k, (bnd, total, n) in work.items()}
    peaks, peak_src = load_peaks()
    traffic = read_traffic()
    kernels = {}
    t_roof_ms = 0.0
    for k, (bound, amount, launches) in work.items():
        ms_launch = per_step[k] / launches
        if bound == "tensor":
            ach = amount / (ms_launch / 1000.0) / 1e12
            peak = peaks["bf16_tflops_sustained"]
            unit = "TFLOP/s"
            t_roof_ms += launches * amount / (peak * 1e12) * 1000.0
        else:
            ach = amount / (ms_launch / 1000.0) / 1e9
            peak = peaks["hbm_gbs"]
            unit = "GB/s"
            t_roof_ms += launches * amount / (peak * 1e9) * 1000.0
        kernels[k] = {"bound": bound, "ms_per_step": round(per_step[k], 4), "launches_per_step": launches,
                      "achieved": round(ach, 2), "unit": unit, "frac": round(ach / peak, 4)}
    dom = max(work, key=lambda k: per_step[k])
    dk = kernels[dom]
    bound, amount, launches = work[dom]
    roofline = {
        "kernel": dom,
        "bound": "tensor" if bound == "tensor" else "hbm",
        "achieved": dk["achieved"],
        "peak": peaks["bf16_tflops_sustained"] if bound == "tensor" else peaks["hbm_gbs"],
        "unit": dk["unit"],
        "frac": dk["frac"],
        # the per-row DRAM traffic was captured on the headline wave
        "traffic": traffic[dom] * R if dom in traffic and args.workload == "grouped" else None,
        "peak_source": f"{peak_src} (MEASURED_PEAKS.json: bf16 sustained / HBM copy)",
        "per_launch_work": amount,
        "step_roof_ms": round(t_roof_ms, 4),
        "step_frac": round(t_roof_ms / ms_per_step, 4),
    }

    # End-to-end through the C ABI with host buffers, synchronised per wave
    # (a search reads each wave's results before it builds the next).
    lat = []
    e2e_start = torch.cuda.Event(enable_timing=True)
    e2e_end = torch.cuda.Event(enable_timing=True)
    for i in range(args.warmup + args.steps):
        if i == args.warmup:
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            e2e_start.record(stream)
        for w in step_waves(i):
            t0 = time.perf_counter()
            w.dstep.buf.copy_(w.dstep.host, non_blocking=True)
            w.run()
            w.host_out.copy_(w.out, non_blocking=True)
            stream.synchronize()
            if i >= args.warmup:
                lat.append(time.perf_counter() - t0)
    e2e_end.record(stream)
    torch.cuda.synchronize()
    e2e_ms = reduce_max(e2e_start.elapsed_time(e2e_end), device)
    e2e = {
        "value": rows_all * args.steps / (e2e_ms / 1000.0),
        "unit": UNIT,
        "h2d_bytes_per_step": int(sum(w.dstep.h2d_bytes for w in step_waves(0))),
        "d2h_bytes_per_step": int(sum(w.host_out.numel() * 4 for w in step_waves(0))),
        "p50_wave_latency_ms": round(1000.0 * statistics.median(lat), 3),
    }
    result.update({
        "value": value,
        "ms_per_step": ms_per_step,
        "passes_ms_per_step": [round(p / args.steps, 4) for p in pass_ms],
        "rows_all": rows_all,
        "e2e": e2e,
        "roofline": roofline,
        "kernels": kernels,
        "gpu_launches": int(args.steps * len(step_waves(0)) * count_launches(dims, plans[0])),
        "wave": extra if args.workload in ("grouped", "d1024") else None,
    })
    del waves, pool
    torch.cuda.synchronize()
    return result


def run_model_api(args, model, dims, device, rank, world):
    """The headline wave through the dense reference-compatible model API
    (``forward_decode_grouped`` with the padded prefix stack the reference's
    merge builds, merged_executors.py:187-196) and through the paged rollout
    executors (imba_chess_b200.executors); each call synchronised."""
    import torch

    from imba_chess_b200 import synth
    from imba_chess_b200.executors import PagedDecodeRequest, make_decode_wave_executor, make_root_eval_executor

    _, wave = workload(args, rank, world)
    lens = wave.prefix_lens
    G, B, L = len(lens), wave.num_rows, dims.num_layers
    tok = synth.concat_tokens(wave.prefix_tokens)
    offsets = np.concatenate([[0], np.cumsum(lens)])
    batch = {k: torch.from_numpy(v) for k, v in tok.items()}
    batch["seq_offsets"] = torch.from_numpy(offsets)
    batch["total_tokens"] = int(offsets[-1])
    kv = model.forward(batch, return_loss=False, return_kv=True)["kv_caches"]
    max_p = max(lens)
    stack = []
    for k, v in kv:  # the reference's per-wave merge: pad every prefix to maxP and stack
        ks = torch.zeros((G, dims.num_heads, max_p, dims.attention_dim), dtype=k.dtype, device=device)
        vs = torch.zeros((G, dims.num_heads, max_p, dims.linear_dim), dtype=v.dtype, device=device)
        for g in range(G):
            a, b = int(offsets[g]), int(offsets[g + 1])
            ks[g, :, : b - a] = k[:, a:b]
            vs[g, :, : b - a] = v[:, a:b]
        stack.append((ks, vs))
    del kv
    rt = wave.row_tokens
    new = {k: torch.from_numpy(v).to(device) for k, v in rt.items()}
    gi = torch.from_numpy(wave.group_index).to(device)
    pos = torch.from_numpy(np.asarray(lens)[wave.group_index]).to(device)
    lens_t = torch.tensor(lens, device=device)

    def call():
        return model.forward_decode_grouped(new_token_batch=new, positions=pos, group_index=gi,
                                            prefix_kv_grouped=stack, prefix_lens=lens_t, prefix_lens_list=lens)

    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    lat = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        call()
        torch.cuda.synchronize()
        lat.append(time.perf_counter() - t0)
    dense_ms = 1000.0 * statistics.median(lat)
    # paged: roots into the pool once, then the decode wave per call
    pool = model.new_pool(sum(-(-n // 16) for n in lens) + (args.warmup + args.steps + 2) * (-(-B // 16) + G) + 64)
    root = make_root_eval_executor(model=model, pool=pool)
    games = [r["game"] for r in root([dict(pt) for pt in wave.prefix_tokens])]
    decode = make_decode_wave_executor(model=model, pool=pool)
    reqs = []
    for g in range(G):
        idx = np.nonzero(wave.group_index == g)[0]
        reqs.append(PagedDecodeRequest(game=games[g], tokens=synth.slice_tokens(rt, idx),
                                       parent_rows=[[] for _ in idx],
                                       legal_ids=[wave.legal_ids[i].tolist() for i in idx]))
    for _ in range(args.warmup):
        decode(reqs)
    plat = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        decode(reqs)
        plat.append(time.perf_counter() - t0)
    paged_ms = 1000.0 * statistics.median(plat)
    return {
        "metric": METRIC, "value": B / (dense_ms / 1000.0), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dense_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": full_config(args, B, world),
        "timing": "wall clock per call (p50), each call synchronised",
        "paged_executor": {"value": B / (paged_ms / 1000.0), "unit": UNIT, "ms_per_step": paged_ms},
    }


def run_b200(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=__import__("datetime").timedelta(seconds=300))

    from imba_chess_b200 import synth
    from imba_chess_b200.model import B200HSTUChessModel

    if args.workload == "d1024":
        dims = synth.D1024
    elif args.workload == "prefill_decode":
        dims = synth.ModelDims(512, 8, 8, max_pos=1024)
    else:
        dims = synth.D512
    sd = synth.make_state_dict(dims, 2, profile="reference")
    model = B200HSTUChessModel(sd, dtype=torch.bfloat16, device=device)
    if args.workload == "model_api":
        line = run_model_api(args, model, dims, device, rank, world)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            emit(line)
        return
    sampler = ClockSampler(local)
    res = measure(args, model, dims, device, rank, world, sampler=sampler)

    line = {
        "metric": METRIC,
        "value": res["value"],
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": res["ms_per_step"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": full_config(args, res["rows_all"], world),
        "e2e": res["e2e"],
        "roofline": res["roofline"],
        "kernels": res["kernels"],
        "clocks": sampler.summary(),
        "gpu_launches": res["gpu_launches"],
        "passes_ms_per_step": res["passes_ms_per_step"],
    }
    if "prefill" in res:
        line["prefill"] = res["prefill"]
    wave = res["wave"]
    # The sequential-halving search rounds (1,024 games per GPU), measured in
    # the same run on the same model (every rank takes the same steps).
    if args.workload == "grouped" and not args.no_halving:
        hargs = workload_args(args, "halving")
        hres = measure(hargs, model, dims, device, rank, world)
        line["halving"] = {
            "value": hres["value"], "unit": UNIT, "ms_per_step": hres["ms_per_step"],
            "passes_ms_per_step": hres["passes_ms_per_step"],
            "config": full_config(hargs, hres["rows_all"], world), "e2e": hres["e2e"],
            "roofline": {k: hres["roofline"][k] for k in ("kernel", "bound", "achieved", "peak", "unit", "frac",
                                                            "step_roof_ms", "step_frac")},
            "gpu_launches": hres["gpu_launches"],
        }
    if rank == 0 and world == 1 and not args.no_service and wave is not None:
        line["service_api"] = service_api(args, dims, wave, sd, device)
    if rank == 0 and world == 1 and not args.no_cpu_baseline and wave is not None:
        cores = os.cpu_count() or 1
        if os.path.isdir(os.path.join(REF_PATH, "imba_chess")):
            n_rows, times = reference_cpu_rate(dims, wave, args.cpu_sample_parents, seconds=args.cpu_seconds)
            line["cpu_baseline"] = {
                "value": n_rows * len(times) / sum(times), "unit": UNIT, "cores": cores, "kind": "reference",
                "sample": f"the wave's first {args.cpu_sample_parents} parents ({n_rows} sibling rows) x "
                          f"{len(times)} waves, reference ActorInferenceServer.service(), fp32 eager torch",
                "cpu_model": cpu_model(), "torch": _torch_version()}
        n_rows, times = cpu_oracle_rate(dims, wave, args.cpu_sample_parents, steps=3)
        port = {"value": n_rows * len(times) / sum(times), "unit": UNIT, "cores": cores, "kind": "port",
                "sample": f"the wave's first {args.cpu_sample_parents} parents ({n_rows} sibling rows) x "
                          f"{len(times)} repetitions, numpy oracle fp32"}
        if "cpu_baseline" in line:
            line["cpu_baseline_port"] = port
        else:
            line["cpu_baseline"] = port
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        emit(line)


def service_api(args, dims, wave, sd, device):
    """Reference-compatible ActorInferenceServer.service() on the same wave:
    one WaveRequest per parent, Python wire objects in and out."""
    import torch

    from imba_chess_b200 import synth
    from imba_chess_b200.model import B200HSTUChessModel
    from imba_chess_b200.protocol import RootEvalRequest, WaveRequest, WaveRow
    from imba_chess_b200.server import ActorInferenceServer

    model = B200HSTUChessModel(sd, dtype=torch.bfloat16, device=device)
    B = wave.num_rows
    reps = 7
    pages = sum(-(-n // 16) for n in wave.prefix_lens) + (reps + 2) * (-(-B // 16) + len(wave.prefix_lens)) + 64
    server = ActorInferenceServer(model=model, device=device, dtype=torch.bfloat16, kv_pool_pages=pages)
    roots = [RootEvalRequest(worker_id=g, turn_id=0, legal_vocab_ids=[2], batch_arrays=synth.root_batch_arrays(pt))
             for g, pt in enumerate(wave.prefix_tokens)]
    server.service(roots)
    reqs = []
    rt = wave.row_tokens
    for g in range(len(wave.prefix_tokens)):
        rows = []
        for i in np.nonzero(wave.group_index == g)[0]:
            bs = {"piece_ids": rt["piece_ids"][i].tolist(), **{k: int(rt[k][i]) for k in SIDE_KEYS}}
            rows.append(WaveRow(node_id=int(i), parent_id=None, prev_move_vocab_id=int(rt["prev_move_id"][i]),
                                board_state=bs, legal_vocab_ids=wave.legal_ids[i].tolist()))
        if rows:
            reqs.append(WaveRequest(worker_id=g, turn_id=0, rows=rows))
    server.service(reqs)  # warm-up
    for k in server.stats:
        server.stats[k] = 0
    lat = []
    for _ in range(reps):
        t0 = time.perf_counter()
        server.service(reqs)
        lat.append(time.perf_counter() - t0)
    p50 = statistics.median(lat)
    st = server.stats
    return {"value": B / p50, "unit": UNIT, "p50_wave_latency_ms": round(1000 * p50, 3), "calls": reps,
            "build_ms_per_wave": round(1000 * st["wave_build_s"] / reps, 3),
            "gpu_ms_per_wave": round(1000 * st["wave_gpu_s"] / reps, 3),
            "post_ms_per_wave": round(1000 * st["wave_post_s"] / reps, 3)}


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
