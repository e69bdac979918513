"""Training-throughput benchmark: Mimir2 dense ~1.3B (24 x 2048, 16 Q / 4 KV heads of 128,
SwiGLU 5632, vocab 65536), seq 4096, 4 sequences per GPU, prefix-LM mask with prompt length
uniform in [0, 2048], FSDP2 bf16 compute / fp32 master weights, AdamATan2 (+EMA).
``--optimizer muon`` is the Muon variant of the same model (5 Newton-Schulz iterations,
coefficients (3.4445, -4.7750, 2.0315), momentum 0.95 on every 2-D hidden matrix; Adam for
embeddings, norms and the head).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--optimizer adam_atan2|muon]

For N > 1 run under ``torch.distributed.run`` (one rank per GPU).  Rank 0 prints one JSON
line.  ``value`` is device-timed (CUDA events around exactly K steps, barrier + synchronize
on both sides, max over ranks) with the step's inputs already on the device; ``e2e`` times
the same K-step loop through the public training-step API including, every step, the
pinned host->device copy of the batch and the device->host read of the loss.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
SEQ_LEN, SEQS_PER_GPU, VOCAB = 4096, 4, 65536
MODEL = dict(n_layers=24, hidden_size=2048, num_heads=16, num_key_value_heads=4, expansion=4.125)
# BASELINE config 3 (``--config moe``): 16 layers, d 2048, 64 experts top-2 of FFN 1408 plus one
# shared expert, expert parallelism over the GPUs, aux-loss-free routing balance, Zipf(1.1) tokens.
MOE = dict(n_layers=16, experts=64, top_k=2, expert_ffn=1408, shared=1, zipf=1.1)
# Router rows are random-initialised in both arms (the reference's zero rows would send every
# token to experts 0 and 1, whatever the data): normal with std 1/sqrt(d).
ROUTER_STD = 2048 ** -0.5
CONFIG = {"name": "dense"}  # set from --config in main()
METRIC = "train tokens/sec (box, device-timed, max over ranks) at 1/2/4/8 B200; MFU"
BASELINE_VALUE = None  # the reference publishes no throughput number
MODEL_LABEL = {"dense": "Mimir2 dense ~1.3B (24x2048, 16Q/4KV heads x128, SwiGLU 5632, vocab 65536)",
               "moe": "Mimir2 MoE (16x2048, 16Q/4KV heads x128, 64 experts top-2 FFN 1408 + 1 shared expert, "
                      "aux-loss-free routing balance, vocab 65536, Zipf(1.1) token ids)"}
OPTIMIZER_LABEL = {"adam_atan2": "AdamATan2 + EMA",
                   "muon": "MuonAdamW + EMA (Muon on 2-D hidden matrices, 5 Newton-Schulz iterations in fp32, "
                           "momentum 0.95; Adam on the rest)"}


def arch_dict(kv_heads=4, reference=False):
    if CONFIG["name"] == "moe":
        base = _arch_base(kv_heads) | dict(n_layers=MOE["n_layers"], moe_num_experts=MOE["experts"],
                                           moe_top_k=MOE["top_k"], moe_sparse=True, moe_aux_loss_free=True)
        if reference:  # no expert width, shared experts or expert parallelism in the reference:
            # its experts are dense-MLP copies; expansion 1.03125 gives 2048*1.03125*2/3 = 1408, which
            # its multiple-of-256 rounding turns into 1536.
            return base | dict(expansion=1.03125)
        return base | dict(moe_expert_intermediate_size=MOE["expert_ffn"], moe_shared_experts=MOE["shared"],
                           moe_dispatch="grouped", moe_expert_parallel=True, moe_router_init_std=ROUTER_STD)
    return _arch_base(kv_heads)


def _arch_base(kv_heads):
    return dict(name="mimir2", max_seq_len=SEQ_LEN, n_layers=MODEL["n_layers"], hidden_size=MODEL["hidden_size"],
                num_heads=MODEL["num_heads"], num_key_value_heads=kv_heads, expansion=MODEL["expansion"],
                init_type="lecun_normal", norm_type="pre", norm_eps=1e-6, pos_emb_type="rope", rope_theta=10000.0,
                recurrence_mode="looped", half_layers=False, H_override={"n_layers": 0}, H_cycles=1, L_cycles=1,
                bp_min_steps=2, bp_max_steps=2, bp_warmup_ratio=0.0, fwd_bwd_dtype="bfloat16", vocab_size=VOCAB)


# ---------------------------------------------------------------------------------------- batch
def synthetic_batch(rank: int, step: int):
    """Host batch in the corpus format: packed inputs/labels/positions + prefix-LM metadata."""
    rng = np.random.default_rng(1_000_003 * rank + step)
    T = SEQ_LEN * SEQS_PER_GPU
    prefix = rng.integers(0, 2049, size=SEQS_PER_GPU).astype(np.int32)
    if CONFIG["name"] == "moe":  # Zipf(s) over the vocabulary skews the routing
        p = np.arange(1, VOCAB + 1, dtype=np.float64) ** -MOE["zipf"]
        p /= p.sum()
        inputs = rng.choice(VOCAB, size=T, p=p).astype(np.int32)
        labels = rng.choice(VOCAB, size=T, p=p).astype(np.int32)
    else:
        inputs = rng.integers(0, VOCAB, size=T).astype(np.int32)
        labels = rng.integers(0, VOCAB, size=T).astype(np.int32)
    for s in range(SEQS_PER_GPU):
        labels[s * SEQ_LEN: s * SEQ_LEN + max(int(prefix[s]) - 1, 0)] = -100  # supervise the answer only
    positions = np.tile(np.arange(SEQ_LEN, dtype=np.int32), SEQS_PER_GPU)
    causal = (SEQ_LEN - prefix).astype(np.int32)
    pad = lambda a: np.pad(a, (0, T - a.shape[0]))
    cu = np.pad(np.cumsum(np.full(SEQS_PER_GPU, SEQ_LEN, np.int32)), (1, T - SEQS_PER_GPU - 1)).astype(np.int32)
    tensors = dict(inputs=inputs, labels=labels, position_ids=positions, prefix_lens=pad(prefix),
                   causal_lens=pad(causal), cu_seqlens=cu)
    scalars = dict(total_seqlen=T, numseqs=SEQS_PER_GPU, max_seqlen_prefix=int(prefix.max()),
                   max_seqlen_causal=int(causal.max()), max_seqlen_all=SEQ_LEN)
    host = {k: torch.from_numpy(v).pin_memory() if torch.cuda.is_available() else torch.from_numpy(v)
            for k, v in tensors.items()}
    return host, scalars


def attention_pairs(host) -> int:
    """Visible (query, key) pairs of the prefix-LM mask in one local batch."""
    total = 0
    for s in range(SEQS_PER_GPU):
        p = int(host["prefix_lens"][s])
        L = SEQ_LEN
        total += p * p + sum(r + 1 for r in range(p, L)) if p < L else p * p
    return total


def model_flops_per_step(host, kv_heads) -> float:
    d, H, hd, F = MODEL["hidden_size"], MODEL["num_heads"], 128, 5632
    layers = MODEL["n_layers"]
    mlp = d * 2 * F + F * d
    if CONFIG["name"] == "moe":  # active experts per token (top-k + shared) and the router
        layers = MOE["n_layers"]
        fe = CONFIG.get("expert_ffn", MOE["expert_ffn"])
        mlp = CONFIG.get("active_experts", MOE["top_k"] + MOE["shared"]) * 3 * d * fe + d * MOE["experts"]
    per_layer = d * (2 * H + 2 * kv_heads) * hd + H * hd * d + mlp
    matmul_params = layers * per_layer + d * VOCAB
    T = SEQ_LEN * SEQS_PER_GPU
    dense = 6.0 * matmul_params * T
    attn_fwd = 4.0 * hd * H * attention_pairs(host) * layers
    return dense + 3.0 * attn_fwd


# ---------------------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        self.path = os.path.join("/tmp", f"mimir_clocks_{os.getpid()}.csv")
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(gpu_index)], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


# ---------------------------------------------------------------------------------------- distributed
def init_distributed(gpus: int):
    if "RANK" not in os.environ:
        if gpus != 1:
            raise SystemExit("--gpus N > 1 must be launched with torch.distributed.run")
        os.environ.update(RANK="0", WORLD_SIZE="1", LOCAL_RANK="0", MASTER_ADDR="127.0.0.1",
                          MASTER_PORT=str(29500 + os.getpid() % 1000))
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    from datetime import timedelta
    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
    return rank, world, local


def device_batch(host, scalars, device, wrap):
    batch = {k: v.to(device, non_blocking=True) for k, v in host.items()}
    batch.update({k: wrap(torch.tensor(v)) for k, v in scalars.items()})
    return batch


def max_over_ranks(x: float) -> float:
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed_loop(run_step, batches, steps: int):
    """CUDA-event time of exactly `steps` calls (inputs already on device), max over ranks."""
    dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    torch.cuda.nvtx.range_push("timed")
    for i in range(steps):
        run_step(batches[i % len(batches)])
    torch.cuda.nvtx.range_pop()
    end.record()
    torch.cuda.synchronize()
    dist.barrier()
    return max_over_ranks(start.elapsed_time(end) / 1000.0)


# ---------------------------------------------------------------------------------------- our arm
def heldout_loss(model_call, device, wrap) -> float:
    """Forward-only loss on a batch no step has seen (step index 10**6).  The timed loop alternates
    two batches, so its training loss falls towards zero as the 1.3B model memorises their random
    labels; on unseen uniform labels the loss must stay near ln(65536) = 11.09."""
    host, scalars = synthetic_batch(dist.get_rank(), 10 ** 6)
    with torch.no_grad():
        metrics = model_call(device_batch(host, scalars, device, wrap))
    return float((metrics["loss"][0] / metrics["loss"][1]).item())


def measure_ours(args, rank, world, local, kv_heads):
    """Build our model with `kv_heads` KV heads, warm up, then time K steps on the device and K
    steps end to end.  Releases the model and its peer buffers before returning."""
    import gc

    from mimir_b200.config.schema import PretrainConfig
    from mimir_b200.models.common import wrap_tensor
    from mimir_b200.ops._ext import launch_count
    from mimir_b200.optim.schedules import update_lr
    from mimir_b200.parallel.replicated import engine_of
    from mimir_b200.train.setup import create_model_and_optimizer, make_train_state
    from mimir_b200.train.steps import train_accumulated_batches

    device = torch.device("cuda", local)
    arch = arch_dict(kv_heads=kv_heads)
    vocab = arch.pop("vocab_size")
    config = PretrainConfig(arch=arch, data=dict(path="synthetic"), global_batch_size=SEQ_LEN * SEQS_PER_GPU * world,
                            epochs=1, lr=3e-4, lr_warmup_steps=0, lr_min_ratio=1.0, weight_decay=0.1, beta1=0.9,
                            beta2=0.95, ema=None if CONFIG["name"] == "moe" else 0.9999,
                            distributed_strategy=args.dp, lr_auto=False,
                            optimizer=args.optimizer, muon_momentum=0.95, muon_ns_steps=5)
    torch.manual_seed(0)
    model, carry, optim = create_model_and_optimizer(config, {"vocab_size": vocab, "max_seq_len": SEQ_LEN}, device)
    state = make_train_state(config, model, carry, optim, total_steps=10_000, device=device)
    hosts = [synthetic_batch(rank, i) for i in range(2)]
    dev_batches = [device_batch(h, s, device, wrap_tensor) for h, s in hosts]

    def step(batch):
        state.step += 1
        update_lr(config, state)
        metrics, _ = train_accumulated_batches(config, rank, state, [batch])
        return metrics

    for i in range(args.warmup):
        step(dev_batches[i % 2])
    torch.cuda.synchronize()
    launches0 = launch_count()
    clocks = ClockSampler(local)
    seconds = timed_loop(step, dev_batches, args.steps)
    clock_info = clocks.stop()
    launches = (launch_count() - launches0) // max(args.steps, 1) * args.steps

    # End to end through the public step API: H2D of each step's batch + D2H of its loss.
    h2d = sum(t.numel() * t.element_size() for t in hosts[0][0].values())
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    losses = []
    for i in range(args.steps):
        host, scalars = hosts[i % 2]
        metrics = step(device_batch(host, scalars, device, wrap_tensor))
        losses.append((metrics["loss"][0] / metrics["loss"][1]).item())
    torch.cuda.synchronize()
    e2e_seconds = max_over_ranks(time.perf_counter() - t0)
    unseen = heldout_loss(lambda b: state.model(batch=b, carry=state.carry, bp_steps=2)[2], device, wrap_tensor)
    from mimir_b200.ops._ext import check_kernel_status
    check_kernel_status(device)  # no kernel wait of the measured steps timed out
    flops = model_flops_per_step(hosts[0][0], kv_heads)
    engine = engine_of(model)
    if engine is not None:
        dist.barrier()
        engine.close()
    del state, model, carry, optim, dev_batches
    gc.collect()
    torch.cuda.empty_cache()
    return dict(seconds=seconds, e2e_seconds=e2e_seconds, h2d=h2d, flops=flops, clocks=clock_info,
                launches=launches, final_loss=losses[-1], heldout_loss=unseen)


def run_ours(args, rank, world, local):
    sys.path.insert(0, ROOT)
    from mimir_b200.ops._ext import ext

    ext()  # fail loudly if the extension is missing
    r = measure_ours(args, rank, world, local, args.kv_heads)
    if args.dp != "replicated":
        label = f"fsdp{world}"
    elif args.optimizer == "muon":
        label = (f"dp{world}: replicated bf16 weights, fp32 master+optimizer state sharded like FSDP2; fused NVLink "
                 "reduce + Adam/momentum + gather-to-owner kernel, Newton-Schulz once per matrix on its owner rank, "
                 "fused scatter + update + all-gather kernel")
    else:
        label = (f"dp{world}: replicated bf16 weights, fp32 master+AdamATan2 state sharded like FSDP2, one fused "
                 "NVLink reduce-scatter+update+all-gather kernel per step")
    if CONFIG["name"] == "moe":
        label += (f"; ep{world}: {MOE['experts'] // world} experts per GPU, token rows dispatched/combined over "
                  "NVLink peer memory (route plan from all-gathered expert counts, no capacity factor)")
    extra = {"final_loss": r["final_loss"], "heldout_loss": r["heldout_loss"], "parallelism": label,
             "num_key_value_heads": args.kv_heads}
    if CONFIG["name"] == "dense" and args.same_config and args.kv_heads != MODEL["num_heads"]:
        # The reference ties KV heads to Q heads, so its arm can only run 16 KV heads; measure our
        # arm on that exact architecture too.
        same = measure_ours(args, rank, world, local, MODEL["num_heads"])
        tokens = SEQ_LEN * SEQS_PER_GPU * world * args.steps
        extra["same_config"] = {
            "num_key_value_heads": MODEL["num_heads"], "value": round(tokens / same["seconds"], 1),
            "ms_per_step": round(same["seconds"] / args.steps * 1000.0, 3),
            "e2e": {"value": round(tokens / same["e2e_seconds"], 1), "unit": "tokens/s"},
            "final_loss": same["final_loss"], "heldout_loss": same["heldout_loss"], "clocks": same["clocks"],
            "gpu_launches": same["launches"],
            "note": "the reference arm's architecture (KV heads = Q heads, its transformer.py:78)"}
    return emit(args, world, r["seconds"], r["e2e_seconds"], r["h2d"], 4, r["flops"], r["clocks"], r["launches"],
                impl="ours", extra=extra)


# ---------------------------------------------------------------------------------------- reference arm
def _stub_missing_reference_deps():
    """The offline wheelhouse lacks `coolname` and `omegaconf`, which the reference's
    training/runtime.py imports at module level for run naming and Hydra config handling.
    Neither is used on the training-step path; empty stand-ins let the unmodified module import."""
    import types
    for name in ("coolname", "omegaconf"):
        try:
            __import__(name)
            continue
        except ImportError:
            pass
        mod = types.ModuleType(name)
        if name == "coolname":
            mod.generate_slug = lambda n=2: "bench-run"
        else:
            mod.DictConfig = dict

            class OmegaConf:  # noqa: D401 - placeholder
                @staticmethod
                def to_container(cfg, **_):
                    return dict(cfg)
            mod.OmegaConf = OmegaConf
        sys.modules[name] = mod


def run_reference(args, rank, world, local):
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "mimir")):
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}))
        return
    sys.path.insert(0, ref)
    _stub_missing_reference_deps()
    from mimir.model import Mimir2 as RefMimir2
    from mimir.model.accelerator import set_accelerator_type
    from mimir.model.adam_atan2 import AdamATan2 as RefAdam
    from mimir.model.common import wrap_tensor
    from mimir.model.lm_head import LMHead as RefHead
    from mimir.training.config import PretrainConfig as RefConfig
    from mimir.training.distributed import apply_fsdp, fsdp_wrap_modules
    from mimir.training.schedules import update_lr
    from mimir.training.state import TrainState
    from mimir.training.steps import train_accumulated_batches

    # FlashAttention-4 (flash_attn.cute) is not installable offline, so the reference's own
    # dense prefix-LM attention backend (accelerator "none") is the path that can run.
    set_accelerator_type("none")
    device = torch.device("cuda", local)
    arch = arch_dict(kv_heads=None, reference=True)  # the reference ties KV heads to Q heads
    arch.pop("num_key_value_heads")
    vocab = arch.pop("vocab_size")
    compiled = os.environ.get("MIMIR_REF_COMPILE", "1") == "1"
    config = RefConfig(arch=arch, data=dict(path="synthetic"), global_batch_size=SEQ_LEN * SEQS_PER_GPU * world,
                       epochs=1, lr=3e-4, lr_warmup_steps=0, lr_min_ratio=1.0, weight_decay=0.1, beta1=0.9, beta2=0.95,
                       ema=None if CONFIG["name"] == "moe" else 0.9999, distributed_strategy="fsdp", accelerator_type="sm100", lr_auto=False,
                       compile_train_batch=compiled)
    model_cfg = config.arch.model_dump() | {"vocab_size": vocab, "max_seq_len": SEQ_LEN} | config.data.model_dump() | {
        "fwd_bwd_dtype": "bfloat16", "activation_checkpointing": "none"}
    torch.manual_seed(0)
    with torch.device(device):
        model = RefHead(RefMimir2(model_cfg), model_cfg)
    if CONFIG["name"] == "moe":  # random router rows, as in our arm (the reference initialises zeros)
        gen = torch.Generator(device=device).manual_seed(1234)
        with torch.no_grad():
            for name, p in model.named_parameters():
                if ".router.rows." in name:
                    p.normal_(0.0, ROUTER_STD, generator=gen)
    for buf in model.buffers():
        dist.broadcast(buf, src=0)
    for module in fsdp_wrap_modules(model, "transformer_block"):
        apply_fsdp(module, torch.bfloat16)
    apply_fsdp(model, torch.bfloat16)
    if args.optimizer == "muon":
        from mimir.model.muon import MuonAdamW as RefMuon
        optim = RefMuon(model.named_parameters(), momentum=0.95, ns_steps=5, muon_lr_scale=1.0, lr=0.0,
                        betas=(0.9, 0.95), weight_decay=0.1, ema=0.9999)
    else:
        optim = RefAdam(model.parameters(), lr=0.0, betas=(0.9, 0.95), weight_decay=0.1,
                        ema=None if CONFIG["name"] == "moe" else 0.9999)
    state = TrainState(model=model, carry=None, optim=optim, step=0, total_steps=10_000, fwd_bwd_dtype=torch.bfloat16,
                       use_cuda_autocast=False)
    hosts = [synthetic_batch(rank, i) for i in range(2)]
    dev_batches = [device_batch(h, s, device, wrap_tensor) for h, s in hosts]

    def step(batch):
        state.step += 1
        update_lr(config, state)
        metrics, _ = train_accumulated_batches(config, rank, state, [batch], config.compile_train_batch,
                                               bp_steps=2)
        return metrics

    for i in range(args.warmup):
        step(dev_batches[i % 2])
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    seconds = timed_loop(step, dev_batches, args.steps)
    clock_info = clocks.stop()
    h2d = sum(t.numel() * t.element_size() for t in hosts[0][0].values())
    dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    losses = []
    for i in range(args.steps):
        host, scalars = hosts[i % 2]
        metrics = step(device_batch(host, scalars, device, wrap_tensor))
        losses.append((metrics["loss"][0] / metrics["loss"][1]).item())
    torch.cuda.synchronize()
    e2e_seconds = max_over_ranks(time.perf_counter() - t0)
    unseen = heldout_loss(lambda b: state.model(batch=b, carry=state.carry, bp_steps=2)[2], device, wrap_tensor)
    if CONFIG["name"] == "moe":
        CONFIG.update(expert_ffn=1536, active_experts=MOE["top_k"])
    flops = model_flops_per_step(hosts[0][0], MODEL["num_heads"])
    extra = {"attention_backend": "reference dense prefix-LM SDPA (FA4 unavailable offline)",
             "num_key_value_heads": MODEL["num_heads"], "torch_compile": compiled, "final_loss": losses[-1],
             "heldout_loss": unseen}
    if CONFIG["name"] == "moe":
        extra["moe_reference_limits"] = ("no expert FFN width option (experts are dense-MLP copies: FFN 1536, the "
                                         "multiple of 256 nearest 1408), no shared expert, no expert parallelism "
                                         "(all 64 experts on every rank)")
    return emit(args, world, seconds, e2e_seconds, h2d, 4, flops, clock_info, None, impl="reference", extra=extra)


# ---------------------------------------------------------------------------------------- output
def emit(args, world, seconds, e2e_seconds, h2d_bytes, d2h_bytes, flops_per_step_per_rank, clocks, launches, impl,
         extra=None):
    tokens = SEQ_LEN * SEQS_PER_GPU * world * args.steps
    value = tokens / seconds
    e2e = tokens / e2e_seconds
    ms = seconds / args.steps * 1000.0
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    achieved = flops_per_step_per_rank / (seconds / args.steps)
    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": (value / BASELINE_VALUE) if BASELINE_VALUE else None, "dtype": "bf16",
        "data": ("synthetic Zipf(1.1) token ids" if CONFIG["name"] == "moe" else "synthetic uniform token ids")
                + ", random-init weights, 2 batches per rank alternated",
        "config": {"model": MODEL_LABEL[CONFIG["name"]],
                   "global_batch": SEQ_LEN * SEQS_PER_GPU * world, "seq_len": SEQ_LEN, "micro_batch": SEQS_PER_GPU,
                   "parallelism": (extra or {}).pop("parallelism", f"fsdp{world}"),
                   "mask": "prefix-LM, prompt length uniform [0,2048]",
                   "optimizer": (OPTIMIZER_LABEL[args.optimizer].replace(" + EMA", "") + " (no EMA)") if CONFIG["name"] == "moe"
                   else OPTIMIZER_LABEL[args.optimizer],
                   "l2": "inputs larger than L2 (weights+activations >> 126 MB)"},
        "mfu": round(achieved / 2.25e15, 4),
        "frac_of_measured_bf16": round(achieved / (peaks.get("bf16_tflops_sustained", 1422.4) * 1e12), 4),
        "clocks": clocks,
        "e2e": {"value": round(e2e, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d_bytes,
                "d2h_bytes_per_step": d2h_bytes},
        "impl": impl,
    }
    if launches is not None:
        out["gpu_launches"] = launches
    if extra:
        out.update(extra)
    if dist.get_rank() == 0:
        print(json.dumps(out), flush=True)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["dense", "moe"], default="dense",
                    help="dense: the headline 1.3B config; moe: the 64-expert MoE config with expert parallelism")
    ap.add_argument("--optimizer", choices=["adam_atan2", "muon"], default="adam_atan2",
                    help="adam_atan2: the headline config; muon: the Muon variant of the same model")
    ap.add_argument("--kv-heads", type=int, default=MODEL["num_key_value_heads"],
                    help="KV heads of our arm's dense model (BASELINE config 2: 4)")
    ap.add_argument("--no-same-config", dest="same_config", action="store_false",
                    help="skip the extra measurement of our arm at the reference's 16 KV heads")
    ap.add_argument("--dp", choices=["replicated", "fsdp"], default="replicated",
                    help="data-parallel engine of our arm (the reference arm always uses its FSDP2)")
    args = ap.parse_args()
    CONFIG["name"] = args.config
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference" and not os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "mimir")):
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref is not installed"}))
        return
    rank, world, local = init_distributed(args.gpus)
    try:
        (run_reference if args.impl == "reference" else run_ours)(args, rank, world, local)
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
