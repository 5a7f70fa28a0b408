"""Headline benchmark: decode tokens/s of Llama-3-8B-architecture serving at TP = N B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 launch one process per GPU:
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

Workload (the Llama-3-8B serving configuration): 64 concurrent streams, 1024-token uniform-random prompts (seed 0),
greedy decoding, random-init bf16 weights of the Llama-3-8B architecture, tensor-parallel over the
N GPUs. All 64 prompts are prefilled first (untimed); then W warm-up decode steps; then:

  * value: K decode steps run by the engine's multi-step decode (CUDA-graph replays with the
    next step's inputs built on the device), timed with CUDA events between barriers, max over
    ranks. Each step reads every weight (16 GB at TP1) and the whole KV history, far more than
    the 126 MB L2, so no flush is needed between steps;
  * e2e: K more decode steps through the public ``Engine.step()`` API, each including the
    host-to-device copy of that step's inputs from pinned memory and the device-to-host read of
    the sampled ids, timed on the host between device synchronisations, max over ranks. The
    engine keeps one step in flight (asynchronous decode: a step is enqueued, its token fed from
    the previous step's sample on the device, before that sample is read back), so the K calls
    enqueue K + 1 steps; ``Engine.flush()`` returns the last one's tokens inside the timed region,
    and the value is the tokens the calls returned over the time.

Rank 0 prints one JSON line.
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

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)

METRIC = "decode tok/s at TP8 (1/2/4/8 GPU); failover pause p99; dead-rank detect ms"

# The baseline: stock vLLM 0.22 (the engine the reference plugs into, unmodified) on the same
# workload, measured by `bench.py --impl stock` on this pool's B200s (tokens/s by GPU count).
STOCK_TOK_S = {1: 12701.7, 2: 18094.9}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def reference_arm(args) -> None:
    why = ("reference cannot be installed offline: its root pyproject is a uv workspace that setuptools "
           "cannot build (flat-layout discovery error), its packages need hatchling (absent from the wheelhouse), "
           "and its engine path is a vLLM 0.31 plugin while vLLM 0.22 is installed")
    ref_dir = os.path.join(HERE, "baseline", "_ref")
    if os.path.isdir(ref_dir) and any(n.startswith("everserve") for n in os.listdir(ref_dir)):
        why = ("reference installed but its decode path is a plugin pinned to vLLM 0.31.0 "
               "(adapters/vllm/PIN); the installed vLLM is 0.22")
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}))


def stock_arm(args) -> None:
    """The stock arm: vLLM (the engine the reference plugs into, unmodified, with none of this
    framework's code) serving the same architecture with dummy random weights, the same 64
    streams of uniform-random 1024-token prompts and greedy decoding, TP over the same GPUs
    (``external_launcher``: one vLLM engine per torchrun rank, in this process). Decode tok/s is
    counted through vLLM's public engine API (``LLMEngine.step``): output tokens gained over K
    steps after W warm-up steps, wall clock between device synchronisations, max over ranks."""
    import tempfile

    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")  # engine core in this process
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    _watchdog(args.deadline, rank)
    import torch

    torch.cuda.set_device(local)
    from transformers import LlamaConfig

    model_dir = tempfile.mkdtemp(prefix="es-stock-")
    LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=500000.0,
                max_position_embeddings=8192, rms_norm_eps=1e-5, tie_word_embeddings=False,
                torch_dtype="bfloat16", architectures=["LlamaForCausalLM"]).save_pretrained(model_dir)
    from vllm import LLM
    from vllm import SamplingParams as VSP
    from vllm.inputs import TokensPrompt

    kw = dict(model=model_dir, load_format="dummy", skip_tokenizer_init=True, tensor_parallel_size=world,
              dtype="bfloat16", max_num_seqs=args.batch, max_model_len=args.prompt_len + args.max_tokens + 16,
              gpu_memory_utilization=0.85, seed=args.seed, enable_prefix_caching=False)
    if world > 1:
        kw["distributed_executor_backend"] = "external_launcher"
    llm = LLM(**kw)
    eng = llm.llm_engine
    g = torch.Generator().manual_seed(args.seed)
    prompts = torch.randint(0, 128256, (args.batch, args.prompt_len), generator=g).tolist()
    sp = VSP(max_tokens=args.max_tokens, temperature=0.0, ignore_eos=True, detokenize=False)
    for i, p in enumerate(prompts):
        eng.add_request(f"s{i}", TokensPrompt(prompt_token_ids=p), sp)
    got: dict[str, int] = {}

    def step() -> None:
        for o in eng.step():
            got[o.request_id] = len(o.outputs[0].token_ids)

    t_pf = time.perf_counter()
    while len(got) < args.batch or min(got.values()) < 1:
        step()
    print(f"[bench stock] prefill of {args.batch}x{args.prompt_len} tokens: {time.perf_counter() - t_pf:.2f} s",
          file=sys.stderr)
    for _ in range(args.warmup):
        step()
    import torch.distributed as dist

    def sync():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    sync()
    before = sum(got.values())
    nvtx = os.environ.get("ES_NVTX") == "1"  # a named range for kernel-list captures of the timed steps
    if nvtx:
        torch.cuda.nvtx.range_push("es_timed")
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    if nvtx:
        torch.cuda.nvtx.range_pop()
    gained = sum(got.values()) - before
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([dt], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    value = gained / dt
    out = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 4), "higher_is_better": True,
           "scaling": "strong", "vs_baseline": 1.0, "dtype": "bf16",
           "data": "synthetic: uniform-random 1024-token prompts (seed 0), vLLM dummy random weights",
           "config": {"model": "Llama-3-8B architecture (32 layers, hidden 4096, 32/8 heads, d 128, ffn 14336, "
                               "vocab 128256)", "global_batch": args.batch, "seq_len": args.prompt_len,
                      "parallelism": f"tp{world}", "engine": f"vLLM {_vllm_version()} (stock, CUDA graphs)",
                      "timing": "wall clock over K LLMEngine.step() calls, output tokens gained"},
           "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": None,
                   "d2h_bytes_per_step": None},
           "gpu_launches": None, "clocks": clk, "impl": "stock"}
    if rank == 0:
        print(json.dumps(out), flush=True)
    os._exit(0)  # vLLM's engine and its process group are torn down by the exit


def _vllm_version() -> str:
    try:
        import vllm

        return vllm.__version__
    except Exception:  # noqa: BLE001
        return "?"


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "stock"])
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt-len", type=int, default=1024)
    ap.add_argument("--max-tokens", type=int, default=512)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--collective", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--sp", action="store_true",
                    help="sequence-parallel decode (token-sliced norms; reduce-scatter and all-gather GEMMs)")
    ap.add_argument("--commit", default="store", choices=["store", "off"],
                    help="store: every step's KV rows and counts are committed to everserve-store (the "
                         "serving configuration); off: no commit (for comparison)")
    ap.add_argument("--deadline", type=float, default=300.0,
                    help="seconds after which a run that has not finished reports a failure and exits")
    args = ap.parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.impl == "stock":
        stock_arm(args)
        return
    assert args.warmup >= 3, "at least 3 warm-up steps"
    assert 4 + args.warmup + 2 * args.steps <= args.max_tokens, "steps exceed the 512-token generation"

    import torch
    import torch.distributed as dist

    from everserve_b200 import _ext
    from everserve_b200.engine import Engine, EngineConfig, LocalExecutor, SamplingParams

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    _watchdog(args.deadline, rank)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    _ext.load()
    collective = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
        from everserve_b200.parallel.collective import make_tp_collective

        collective = make_tp_collective(dev, kind=args.collective)

    max_len = args.prompt_len + args.max_tokens + 16
    block_size = 16
    num_blocks = args.batch * (-(-max_len // block_size)) + 64
    cfg = EngineConfig(args.model, device=str(dev), max_batch=args.batch, max_model_len=max_len,
                       max_prefill_tokens=8192, tensor_parallel=world, seed=args.seed, num_blocks=num_blocks,
                       block_size=block_size, sequence_parallel=args.sp and world > 1)
    ex = LocalExecutor(cfg, rank=rank, collective=collective)
    connector = None
    store = None
    if args.commit == "store":
        store, connector = _store_connector(ex, rank, local, num_blocks * block_size, block_size,
                                            os.environ.get("MASTER_PORT", "0"), world)
    eng = Engine(cfg, executor=ex, connector=connector)
    g = torch.Generator().manual_seed(args.seed)
    vocab = cfg.model.vocab
    prompts = torch.randint(0, vocab, (args.batch, args.prompt_len), generator=g).tolist()
    for p in prompts:
        eng.add_request(p, SamplingParams(max_tokens=args.max_tokens))
    # prefill everything (untimed)
    t_pf = time.perf_counter()
    while eng.scheduler.waiting:
        eng.step()
    torch.cuda.synchronize()
    print(f"[bench] prefill of {args.batch}x{args.prompt_len} tokens: {time.perf_counter() - t_pf:.2f} s",
          file=sys.stderr)
    runner = ex.worker.runner
    for _ in range(args.warmup):
        eng.step()
    torch.cuda.synchronize()
    _check_status(ex, rank, "warm-up")

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # warm the multi-step path once (graph already captured; decode_loop allocations)
    eng.decode_steps(2)
    torch.cuda.synchronize()

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    nvtx = os.environ.get("ES_NVTX") == "1"  # a named range for kernel-list captures of the timed steps
    if nvtx:
        torch.cuda.nvtx.range_push("es_timed")
    start.record()
    eng.decode_steps(args.steps)
    if connector is not None:
        connector.ckv.join_stream()  # the timed region covers every step's KV gather
    end.record()
    if nvtx:
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    dev_ms = max_over_ranks(start.elapsed_time(end))

    # end to end through Engine.step(): H2D of inputs + D2H of sampled ids every step
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    delivered = 0  # tokens the calls returned to the host
    for _ in range(args.steps):
        delivered += sum(1 for _, tok, _ in eng.step() if tok is not None)
    # with a decode step in flight (asynchronous decode) its tokens come back by flush()
    delivered += sum(1 for _, tok, _ in eng.flush() if tok is not None)
    if connector is not None:
        connector.drain()  # every commit of the region acknowledged by the store
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    clk = clocks.stop()

    _check_status(ex, rank, "timed steps")
    # kernel launches of this framework per decode step: count the extension calls of one step
    launches_per_step = count_launches(eng, ex)

    tokens = args.batch * args.steps
    value = tokens / (dev_ms / 1e3)
    e2e = delivered / e2e_s
    out = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(dev_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": round(value / STOCK_TOK_S[world], 4) if world in STOCK_TOK_S else None,
        "dtype": "bf16",
        "data": "synthetic: uniform-random 1024-token prompts (seed 0), random-init weights",
        "config": {"model": "Llama-3-8B architecture (32 layers, hidden 4096, 32/8 heads, d 128, ffn 14336, "
                            "vocab 128256)", "global_batch": args.batch, "seq_len": args.prompt_len,
                   "parallelism": f"tp{world}" + ("-sp" if args.sp and world > 1 else ""),
                   "collective": args.collective if world > 1 else "none",
                   "l2": "inputs larger than L2 (16 GB of weights / TP and the KV history read every step)"},
        "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": runner.h2d_bytes,
                "d2h_bytes_per_step": args.batch * 8},
        "commit": _commit_summary(connector, args),
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk,
        "impl": "ours",
        "so": os.path.basename(_ext.so_path() or ""),
    }
    if rank == 0:
        print(json.dumps(out), flush=True)
    # graphs that hold NCCL calls go before the process group, or its teardown waits for them
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local])
    eng.shutdown()
    if connector is not None:
        connector.close()
    if store is not None:
        store.terminate()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def _store_connector(ex, rank: int, local: int, slots: int, block_size: int, tag: str, world: int):
    """Start the node's everserve-store (the first process of the node) and give this rank a KV
    connector committing to it, as a serving rank does."""
    import shutil

    from everserve_b200.state.connector import StoreConnector
    from everserve_b200.state.kvcopy import PagedKV
    from everserve_b200.state.mirror import MirrorClient, MirrorCommittedKV

    base = "/dev/shm" if shutil.disk_usage("/dev/shm").free > (64 << 30) else "/tmp"
    root = os.path.join(base, f"es-bench-{tag}")
    sock = os.path.join(root, "store.sock")
    proc = None
    if local == 0:
        shutil.rmtree(root, ignore_errors=True)
        os.makedirs(os.path.join(root, "data"), exist_ok=True)
        binary = os.path.join(HERE, "cpp", "bin", "everserve-store")
        if not os.path.exists(binary):
            subprocess.run(["make", "-C", os.path.join(HERE, "cpp"), f"-j{os.cpu_count() or 8}"], check=True,
                           stdout=subprocess.DEVNULL)
        proc = subprocess.Popen([binary, "--socket", f"unix:{sock}", "--data-dir", os.path.join(root, "data"),
                                 "--slots", str(slots), "--budget-bytes", str(256 << 30)],
                                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
    t0 = time.monotonic()
    while not os.path.exists(sock):
        if time.monotonic() - t0 > 60:
            raise RuntimeError(f"everserve-store did not come up at {sock}")
        time.sleep(0.05)
    w = ex.worker
    kv = PagedKV("heads_blocked", w.num_blocks, block_size, w.model.hkv, w.model.d)
    ckv = MirrorCommittedKV(MirrorClient(f"unix:{sock}"), "bench", rank, w.runner.caches, kv, store_slots=slots)
    return proc, StoreConnector(ckv, block_size)


def _commit_summary(connector, args) -> dict:
    if connector is None:
        return {"mode": "off"}
    st = connector.ckv.stats()
    return {"mode": "everserve-store, every step (gather on a side stream, fence 2 steps back)",
            "commits": connector.commits, "bytes": st.get("bytes", 0), "fence_waits": st.get("fence_waits", 0)}


def _fail(rank: int, why: str, code: int) -> None:
    if rank == 0:
        print(json.dumps({"metric": METRIC, "error": why, "impl": "ours"}), flush=True)
    print(f"[bench] rank {rank}: {why}", file=sys.stderr, flush=True)
    os._exit(code)


def _watchdog(deadline_s: float, rank: int) -> None:
    """A run that has not finished by the deadline reports it and exits (a peer that stopped
    answering must not keep every GPU of the job waiting)."""
    import threading

    def fire():
        _fail(rank, f"no result within {deadline_s:.0f} s", 3)

    t = threading.Timer(deadline_s, fire)
    t.daemon = True
    t.start()


def _check_status(ex, rank: int, where: str) -> None:
    """A bounded wait that ran out leaves a status word; a run with one is not a measurement."""
    st = ex.worker.model.ops.check_status()
    coll = getattr(ex.worker.tp, "collective", None)
    cst = coll.status() if coll is not None and hasattr(coll, "status") else 0
    if st or cst:
        late = coll.late_rows() if coll is not None and hasattr(coll, "late_rows") else []
        _fail(rank, f"a bounded wait ran out during {where} (kernel status {st}, collective status {cst}, "
                    f"late rows {late})", 4)


def count_launches(eng, ex) -> int:
    """Kernel launches of the extension in one decode step (the step run eagerly, outside timing)."""
    ops = ex.worker.model.ops
    C = ops.C
    counts = {"n": 0}
    # the bindings that launch kernels of this framework, with the launches of one call (the split
    # decode attention is the attention kernel and its merge); the others (sizes, plans, buffers,
    # switches) launch nothing
    launches = {"rmsnorm": 1, "rope_kv_write": 1, "silu_mul": 1, "embed": 1, "argmax": 1, "sample": 1,
                "decode_advance": 1, "gemm_bf16": 1, "paged_decode": 2, "gemm_silu": 1, "gemm_rope": 1,
                "quant_fp8": 1, "gemm_fp8": 1, "paged_prefill": 1, "moe_route": 1, "moe_topk": 1, "moe_dispatch": 1,
                "moe_ready": 1, "moe_combine": 1, "fdar": 1, "gemm_allreduce": 1, "gemm_allgather": 1,
                "kv_gather": 1, "kv_scatter": 1}

    class Counting:
        def __getattr__(self, name):
            fn = getattr(C, name)
            if not callable(fn) or name not in launches:
                return fn

            def wrapped(*a, **k):
                counts["n"] += launches[name]
                return fn(*a, **k)

            return wrapped

    coll = getattr(ex.worker.tp, "collective", None)
    ops.C = Counting()
    if coll is not None and hasattr(coll, "count_launches"):
        coll.count_launches(counts)
    runner = ex.worker.runner
    saved, saved_async = runner.use_graphs, eng.async_decode
    runner.use_graphs = False
    eng.flush()
    eng.async_decode = False  # one step, not one step and the next enqueued behind it
    try:
        eng.step()
    finally:
        runner.use_graphs = saved
        eng.async_decode = saved_async
        ops.C = C
        if coll is not None and hasattr(coll, "count_launches"):
            coll.count_launches(None)
    return counts["n"] + 1  # + the on-device input advance of multi-step decode


if __name__ == "__main__":
    main()
