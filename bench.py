"""Benchmark: generated tokens/s of the speculative round on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl engine|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

Workload: SmolLM2-1.7B-architecture target (hidden 2048, 24
layers, 32/32 heads, MLP 8192, vocab 49152, RoPE theta 130000, tied) and SmolLM2-135M-
architecture draft (576, 30 layers, 9/3 heads, MLP 1536), both random-init N(0, 0.02) in fp32
then cast to bf16 (no checkpoints: synthetic weights), one 512-token uniform-random prompt
per GPU, k = 4, greedy, 256 new tokens, paged KV block size 16. A step is one
spec.loop.generate() call over the GPU's request (prefill, first token, rounds until 256
tokens); requests are independent, so N GPUs run N requests with no collective in the timed
region (weak scaling) and gather tokens and statistics over NCCL afterwards.

Reported: `value` = generated tokens / device time (CUDA events on the launching stream,
max over ranks); `e2e` = the same tokens / host wall time of the public generate() call,
prompts and outputs as host lists (H2D of the prompt and per-round inputs, D2H of per-round
results inside the timed region); `roofline` = the verify step (the (k+1)-token target
forward, replayed from a CUDA graph) against measured HBM bandwidth, algorithmic bytes =
bf16 weights read once (3,422,752,768 B) + 196,608 B of KV per cached token; `accept` = the
fused accept kernel on BASELINE config 3 (B=64, k=4, V=49152, 113,246,208 B of logits, L2
flushed between launches); `cpu_baseline` = the CPU oracle (numpy restatement of the
reference path) timed on this host on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
REF_INSTALL = ROOT / "baseline" / "_ref"


def _reference_arm_requested(argv: list[str]) -> bool:
    for i, a in enumerate(argv):
        if a == "--impl" and i + 1 < len(argv):
            return argv[i + 1] == "reference"
        if a.startswith("--impl="):
            return a.split("=", 1)[1] == "reference"
    return False


# The reference arm imports the unmodified reference (installed under baseline/_ref), whose
# top-level packages (spec, cache, lm, bench, baselines) share names with the engine's; it
# never imports the engine. Otherwise the engine's package directory comes first (its `bench`
# package, the latency harness, must win over this file).
REFERENCE_ARM = _reference_arm_requested(sys.argv[1:])
if REFERENCE_ARM:
    sys.path[:0] = ([str(REF_INSTALL)] if REF_INSTALL.is_dir() else []) + [str(ROOT)]
else:
    sys.path[:0] = [str(ROOT / "speculative-decoder_b200"), str(ROOT)]

import numpy as np  # noqa: E402
import torch  # noqa: E402

TARGET = dict(hidden_size=2048, num_hidden_layers=24, num_attention_heads=32, num_key_value_heads=32,
              intermediate_size=8192, vocab_size=49152, rope_theta=130000.0, max_position_embeddings=8192)
DRAFT = dict(hidden_size=576, num_hidden_layers=30, num_attention_heads=9, num_key_value_heads=3,
             intermediate_size=1536, vocab_size=49152, rope_theta=100000.0, max_position_embeddings=8192)
PROMPT_LEN, NEW_TOKENS, K, BLOCK = 512, 256, 4, 16
WEIGHT_BYTES = 3_422_752_768          # 1.7B linears + tied embedding, bf16, read once per verify
KV_BYTES_PER_TOKEN = 196_608          # 24 layers x 2 x 32 heads x 64 x 2 B
ACCEPT_BYTES = 113_246_208            # config 3: 64 x (5 + 4) x 49152 x 4 B
# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per algorithmic byte of one verify
# forward, from an ncu capture of the 6-layer case (1.0383 GB of algorithmic bytes): 1.0427 GB
# (profiles/traffic_verify_step_1p7b_6layers_perlayer.txt). Traffic grows with the layers
# streamed, so the full-size figure scales by the same ratio.
VERIFY_TRAFFIC_RATIO = {"layers": (1_046_855_168 + 181_760) / 1_038_340_096}


# BASELINE configs as bench workloads (requests per GPU; requests are independent, so N GPUs
# run N times the requests with no collective in the timed region: weak scaling).
WORKLOADS = {
    2: dict(name="config2", B=1, prompt=PROMPT_LEN, new=NEW_TOKENS, k=K, T=0.0, block=BLOCK, drafter="model",
            prompts="uniform",
            metric="generated tokens/s, 1.7B target k=4 @B1 (config 2, 135M draft, greedy)",
            workload="config2: 1.7B-arch target + 135M-arch draft, bf16 random init, B=1 per GPU, prompt 512, k=4, "
                     "greedy, 256 new tokens, block 16"),
    4: dict(name="config4", B=32, prompt=1024, new=128, k=8, T=0.8, block=16, drafter="model", prompts="uniform",
            metric="generated tokens/s, 1.7B target k=8 T=0.8 @B32 per GPU (config 4, 135M draft)",
            workload="config4: 1.7B-arch target + 135M-arch draft, bf16 random init, 32 requests per GPU (256 over "
                     "8 GPUs), 1024-token uniform prompts, k=8, T=0.8 sampling, 128 new tokens, block 16"),
    5: dict(name="config5", B=4, prompt=8192, new=256, k=6, T=0.0, block=32, drafter="ngram", prompts="segments",
            metric="generated tokens/s, 1.7B target n-gram k=6 @8k context, 4 requests per GPU (config 5)",
            workload="config5: 1.7B-arch target bf16 random init, n-gram drafter (max_n 3), 4 requests per GPU "
                     "(32 over 8 GPUs), 8192-token prompts of 64-id segments each repeated with p=0.5, k=6, greedy, "
                     "256 new tokens, block 32"),
}
NOISY_SIGMA = 0.06  # config 2b: N(0, sigma^2) on the target's logits; sigma 0.06 measured 0.61 acceptance (0.09: 0.49)


def workload_prompts(w: dict, first: int, n: int) -> list[list[int]]:
    """Requests first .. first + n - 1 of a workload, each from its own seed (1000 + index):
    uniform-random ids, or (config 5) 64-id uniform segments each followed by a copy of itself
    with probability 0.5, cut to the prompt length."""
    out = []
    for i in range(first, first + n):
        g = torch.Generator().manual_seed(1000 + i)
        if w["prompts"] == "uniform":
            out.append(torch.randint(0, TARGET["vocab_size"], (w["prompt"],), generator=g).tolist())
            continue
        ids: list[int] = []
        while len(ids) < w["prompt"]:
            seg = torch.randint(0, TARGET["vocab_size"], (64,), generator=g).tolist()
            ids += seg
            if float(torch.rand(1, generator=g)) < 0.5:
                ids += seg
        out.append(ids[: w["prompt"]])
    return out


def weight_bytes(spec: dict) -> int:
    """bf16 bytes of every weight read once per forward: linears, RMSNorm weights and the tied
    embedding/head (3,422,752,768 B for the 1.7B architecture)."""
    H, L, I, V = spec["hidden_size"], spec["num_hidden_layers"], spec["intermediate_size"], spec["vocab_size"]
    d = H // spec["num_attention_heads"]
    qkv = H * (spec["num_attention_heads"] + 2 * spec["num_key_value_heads"]) * d
    per_layer = qkv + spec["num_attention_heads"] * d * H + 3 * H * I
    return 2 * (L * per_layer + V * H + (2 * L + 1) * H)


def kv_bytes_per_token(spec: dict) -> int:
    d = spec["hidden_size"] // spec["num_attention_heads"]
    return spec["num_hidden_layers"] * 2 * spec["num_key_value_heads"] * d * 2


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def make_model(spec: dict, seed: int, device):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=spec["vocab_size"], hidden_size=spec["hidden_size"],
                      intermediate_size=spec["intermediate_size"], num_hidden_layers=spec["num_hidden_layers"],
                      num_attention_heads=spec["num_attention_heads"], num_key_value_heads=spec["num_key_value_heads"],
                      max_position_embeddings=spec["max_position_embeddings"], rms_norm_eps=1e-5,
                      rope_parameters={"rope_type": "default", "rope_theta": spec["rope_theta"]},
                      tie_word_embeddings=True, initializer_range=0.02, attn_implementation="sdpa")
    torch.manual_seed(seed)
    with torch.device(device):
        model = LlamaForCausalLM(cfg)
    return model.to(torch.bfloat16).eval()


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    def __init__(self, index: int) -> None:
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait()

    def summary(self) -> dict:
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def time_verify_step(target, cache_cls, device, context_len: int, reps: int = 30, trace: bool = False,
                     B: int = 1, k: int = K, block: int = BLOCK) -> dict:
    """The (k+1)-token target forward of one round for B rows with `context_len` cached tokens
    each, captured in a CUDA graph and replayed; CUDA events on the replay stream."""
    from specb200.engine import engine_for

    eng = engine_for(target)
    per_row = -(-(context_len + 64) // block)
    cache = cache_cls.for_model(target.config, num_blocks=B * per_row + 4, block_size=block, dtype=torch.bfloat16,
                                device=device)
    rows = list(range(B))
    for r in rows:
        cache.add(r)
    cache.reserve(rows, [context_len - 1] * B)
    past = cache.length(0)
    cache.reserve(rows, [k + 1] * B)
    cap = context_len + 64
    table = torch.zeros(B, -(-cap // block), dtype=torch.int32, device=device)
    for r in rows:
        blocks = cache.tables[r].blocks
        table[r, : len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
    ids = torch.randint(0, TARGET["vocab_size"], (B, k + 1), dtype=torch.int32, device=device)
    n_new = torch.full((B,), k + 1, dtype=torch.int32, device=device)
    pastt = torch.full((B,), past, dtype=torch.int32, device=device)
    logits = torch.empty(B, k + 1, TARGET["vocab_size"], dtype=torch.float32, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    ws = torch.zeros(eng.workspace_bytes(B, k + 1, cap), dtype=torch.uint8, device=device)
    run = lambda: eng.forward_device(cache, ids, n_new, pastt, table, cap, False, logits, status, ws)  # noqa: E731
    run()
    torch.cuda.synchronize()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        run()
    torch.cuda.current_stream(device).wait_stream(side)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(reps):
        g.replay()
    en.record()
    en.synchronize()
    ms = st.elapsed_time(en) / reps
    assert int(status.item()) == 0
    kv_tokens = past + k + 1
    spec = dict(TARGET, num_hidden_layers=target.config.num_hidden_layers)
    r = {"us": ms * 1e3, "bytes": weight_bytes(spec) + B * kv_bytes_per_token(spec) * kv_tokens, "context": kv_tokens,
         "rows": B, "tokens_per_row": k + 1, "layers": spec["num_hidden_layers"]}
    if trace:
        tr = torch.zeros(5 * spec["num_hidden_layers"] + 1, 512, 8, dtype=torch.int64, device=device)
        eng.forward_device(cache, ids, n_new, pastt, table, cap, False, logits, status, ws, trace=tr)
        torch.cuda.synchronize()
        r["trace"] = gemm_trace_summary(tr, spec["num_hidden_layers"])
    return r


def attention_trace(trace: torch.Tensor, base: int, n_layers: int, qkv_end: list, o_r0: list) -> dict:
    """Per-layer attention records ([n_layers][512][8] from `base` in the flat trace): medians
    over layers of the gap after q/k/v (`gap_in`), the gap before o (`gap_out`) and the latest
    offset of each stamp 2..6 from the first wait return (cluster kernel: keys landed, products
    done, warps merged, cluster merged, end; split items: keys landed, merged, published, end)."""
    flat = trace.flatten()
    keys = {k: [] for k in ("gap_in", "gap_out", "entry", "late", "s2", "s3", "s4", "s5", "s6", "ctas")}
    for l in range(n_layers):
        a = flat[base + l * 512 * 8: base + (l + 1) * 512 * 8].view(512, 8).cpu().to(torch.float64)
        ok = a[:, 0] > 0
        if not bool(ok.any()):
            continue
        a = a[ok] / 1e3
        r0 = float(a[:, 1][a[:, 1] > 0].min())
        last = float(a[:, 2:7].max())
        keys["ctas"].append(int(ok.sum()))
        keys["entry"].append(float((a[:, 0] - r0).median()))
        keys["late"].append(int((a[:, 0] > r0).sum()))
        if qkv_end[l] is not None:
            keys["gap_in"].append(r0 - qkv_end[l])
        if l < len(o_r0) and o_r0[l] is not None:
            keys["gap_out"].append(o_r0[l] - last)
        for k in range(2, 7):
            v = a[:, k][a[:, k] > 0]
            if v.numel():
                keys[f"s{k}"].append(float((v - r0).max()))
    return {k: round(statistics.median(v), 2) for k, v in keys.items() if v}


def gemm_trace_summary(trace: torch.Tensor, n_layers: int) -> dict:
    """The per-layer schedule's tensor-core GEMM record ([4 n_layers + 1][512][8] globaltimer
    stamps per CTA: entry, wait return, first stage at the MMA warp, accumulator ready, end,
    normalised operand built (GEMMs with the RMSNorm folded in); GEMMs q/k/v, o, gate/up, down
    per layer, then the LM head). Per GEMM, medians over layers (us) of: `gap`, previous GEMM's
    last end to this one's first wait return (it spans any RMSNorm launch, and for o the
    attention launch); `late`, CTAs that entered after that first wait return; `entry`,
    `first`, `xhat`, `acc`, `endo`: median / max over CTAs of each stamp's offset from the first
    wait return; `body`: first wait return to last end."""
    n = 4 * n_layers + 1
    t = trace.flatten()[: n * 512 * 8].view(n, 512, 8).cpu().to(torch.float64)
    per = []
    for i in range(n):
        ok = t[i, :, 0] > 0
        if not bool(ok.any()):
            per.append(None)
            continue
        ti = t[i][ok] / 1e3
        r0 = float(ti[:, 1][ti[:, 1] > 0].min())
        rec = {"n": int(ok.sum()), "r0": r0, "end": float(ti[:, 4].max()),
               "late": int((ti[:, 0] > r0).sum())}
        for k, key in ((0, "entry"), (2, "first"), (3, "acc"), (4, "endo"), (5, "fenced"), (6, "ticket"),
                       (7, "reduced")):
            v = ti[:, k][ti[:, k] > 0] - r0
            rec[key] = (float(v.median()), float(v.max())) if v.numel() else None
        per.append(rec)
    if per[0] is None:
        return {}
    done = [x for x in per if x is not None]
    out = {"total_us": round(done[-1]["end"] - per[0]["r0"], 1)}
    med = lambda v: round(statistics.median(v), 2)  # noqa: E731
    for j, name in enumerate(["qkv", "o", "gate_up", "down", "head"]):
        rows = [n - 1] if name == "head" else [4 * l + j for l in range(n_layers)]
        rows = [i for i in rows if per[i] is not None]
        if not rows:
            continue
        d = {"ctas": per[rows[0]]["n"], "late": med([per[i]["late"] for i in rows])}
        gaps = [per[i]["r0"] - per[i - 1]["end"] for i in rows if i > 0 and per[i - 1] is not None]
        d["gap"] = med(gaps) if gaps else None
        d["body"] = med([per[i]["end"] - per[i]["r0"] for i in rows])
        for key in ("entry", "first", "acc", "fenced", "ticket", "reduced", "endo"):
            if all(per[i][key] is not None for i in rows):
                d[key] = [med([per[i][key][0] for i in rows]), med([per[i][key][1] for i in rows])]
        out[name] = d
    att = attention_trace(trace, n * 512 * 8, n_layers, [p["end"] if p else None for p in per[0::4]],
                          [p["r0"] if p else None for p in per[1::4]])
    if att:
        out["attention"] = att
    return out


def gemv_trace_summary(trace: torch.Tensor, n_layers: int) -> dict:
    """The GEMV schedule's per-CTA launch record ([4 n_layers + 1][296][8] globaltimer stamps:
    entry, return from griddepcontrol.wait, inputs staged, first weight chunk landed, end; 4
    linear launches per layer, then the LM head). Per linear, medians over layers (us) of:
    `gap`, previous launch's last end to this launch's first wait return (for o it spans the
    attention kernel); `late`, CTAs that entered after that first wait return; `staged`,
    `landed`, `endo`: median / max over CTAs of each stamp's offset from the first wait return;
    `wait`, `dot`: median / max over CTAs of the time spent waiting for weight chunks and in the
    dot products. `attention`: medians over layers of the attention launch's gap after q/k/v
    (`gap_in`) and before o (`gap_out`) and of its stamps' latest offsets from its first wait
    return (keys landed, merged within the CTA, partial published, end of the merge)."""
    n = 4 * n_layers + 1
    t = trace.flatten()[: n * 296 * 8].view(n, 296, 8).cpu().to(torch.float64)
    per = []
    for i in range(n):
        ok = t[i, :, 0] > 0
        if not bool(ok.any()):  # a launch that wrote no record
            per.append(None)
            continue
        ti = t[i][ok] / 1e3
        r0 = float(ti[:, 1].min())
        per.append({"n": int(ok.sum()), "r0": r0, "end": float(ti[:, 4].max()),
                    "late": int((ti[:, 0] > r0).sum()),
                    "staged": (float((ti[:, 2] - r0).median()), float((ti[:, 2] - r0).max())),
                    "landed": (float((ti[:, 3] - r0).median()), float((ti[:, 3] - r0).max())),
                    "endo": (float((ti[:, 4] - r0).median()), float((ti[:, 4] - r0).max())),
                    "wait": (float(ti[:, 5].median()), float(ti[:, 5].max())),
                    "dot": (float(ti[:, 6].median()), float(ti[:, 6].max()))})
    done = [x for x in per if x is not None]
    if per[0] is None:
        return {}
    out = {"total_us": round(done[-1]["end"] - per[0]["r0"], 1)}
    med = lambda v: round(statistics.median(v), 2)  # noqa: E731
    for j, name in enumerate(["qkv", "o", "gate_up", "down", "head"]):
        rows = [n - 1] if name == "head" else [4 * l + j for l in range(n_layers)]
        if any(per[i] is None or (i > 0 and per[i - 1] is None) for i in rows):
            continue
        d = {"ctas": per[rows[0]]["n"], "late": med([per[i]["late"] for i in rows])}
        gaps = [per[i]["r0"] - per[i - 1]["end"] for i in rows if i > 0]
        d["gap"] = med(gaps) if gaps else None
        for key in ("staged", "landed", "endo", "wait", "dot"):
            d[key] = [med([per[i][key][0] for i in rows]), med([per[i][key][1] for i in rows])]
        out[name] = d
    # attention launches (after the linear records)
    att = attention_trace(trace, n * 296 * 8, n_layers, [p["end"] if p else None for p in per[0::4]],
                          [p["r0"] if p else None for p in per[1::4]])
    if att:
        out["attention"] = att
    return out


def time_draft_step(draft, cache_cls, device, context_len: int, reps: int = 30, trace: bool = False,
                    tokens: int = 1) -> dict:
    """One draft-model forward (135M architecture, B=1) of `tokens` new tokens, CUDA graph: 1 as
    in draft steps 1..k-1 of a round, 2 as in step 0 (the token the previous round emitted and
    the one before it when the draft lags)."""
    from specb200.engine import engine_for

    eng = engine_for(draft)
    cache = cache_cls.for_model(draft.config, num_blocks=(context_len + 64) // BLOCK + 4, block_size=BLOCK,
                                dtype=torch.bfloat16, device=device)
    cache.add(0)
    past = cache.reserve([0], [context_len])[0]
    cap = context_len + 64
    table = torch.zeros(1, -(-cap // BLOCK), dtype=torch.int32, device=device)
    blocks = cache.tables[0].blocks
    table[0, : len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
    ids = torch.randint(0, DRAFT["vocab_size"], (1, tokens), dtype=torch.int32, device=device)
    one = torch.full((1,), tokens, dtype=torch.int32, device=device)
    pastt = torch.tensor([context_len - tokens], dtype=torch.int32, device=device)
    logits = torch.empty(1, DRAFT["vocab_size"], dtype=torch.float32, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    ws = torch.zeros(eng.workspace_bytes(1, tokens, cap), dtype=torch.uint8, device=device)
    run = lambda: eng.forward_device(cache, ids, one, pastt, table, cap, True, logits, status, ws)  # noqa: E731
    run()
    torch.cuda.synchronize()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        run()
    torch.cuda.current_stream(device).wait_stream(side)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(reps):
        g.replay()
    en.record()
    en.synchronize()
    del past
    spec = dict(DRAFT, num_hidden_layers=draft.config.num_hidden_layers)
    r = {"us": st.elapsed_time(en) / reps * 1e3,
         "bytes": weight_bytes(spec) + kv_bytes_per_token(spec) * context_len, "context": context_len,
         "layers": spec["num_hidden_layers"]}
    if trace and eng.schedule(1, tokens) == "gemv":
        L = spec["num_hidden_layers"]
        tr = torch.zeros((4 * L + 1) * 296 * 8 + L * 512 * 8, dtype=torch.int64, device=device)
        eng.forward_device(cache, ids, one, pastt, table, cap, True, logits, status, ws, trace=tr)
        torch.cuda.synchronize()
        r["trace"] = gemv_trace_summary(tr, spec["num_hidden_layers"])
    return r


def time_accept(device, reps: int = 20) -> dict:
    """BASELINE config 3 through the fused kernels in logit mode at T = 1, replayed from a CUDA
    graph (so host-side argument handling is not timed), L2 flushed between launches (the
    113 MB of inputs fit in the 126 MB L2): a 256 MB buffer is written, then a second 256 MB
    buffer is read, so that the flush's dirty lines are written back before the timed launch
    instead of during it."""
    from specb200 import ops

    B, V = 64, 49152
    g = torch.Generator(device=device).manual_seed(3)
    pl = torch.randn(B, K + 1, V, generator=g, device=device) * 3.0
    ql = pl[:, :K] + torch.randn(B, K, V, generator=g, device=device)
    draft = torch.multinomial(torch.softmax(ql, -1).reshape(-1, V), 1, generator=g).reshape(B, K)
    ua, ur = torch.rand(B, K, generator=g, device=device), torch.rand(B, generator=g, device=device)
    out = (torch.empty(B, dtype=torch.int64, device=device), torch.empty(B, dtype=torch.int64, device=device))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    clean = torch.ones(64 << 20, dtype=torch.float32, device=device)
    for _ in range(3):
        ops.accept(pl, ql, draft, ua, ur, logits=True, temperature=1.0, check=False, out=out)
    torch.cuda.synchronize()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        ops.accept(pl, ql, draft, ua, ur, logits=True, temperature=1.0, check=False, out=out)
    torch.cuda.current_stream(device).wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        flush.fill_(1)
        clean.sum()
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record()
        graph.replay()
        en.record()
        en.synchronize()
        times.append(st.elapsed_time(en))
    return {"us": statistics.median(times) * 1e3, "bytes": ACCEPT_BYTES}


def request_latency(target, draft, prompts, device, blocks: int, repeats: int = 3) -> dict:
    """TTFT / TPOT / end-to-end of whole generate() requests through the latency harness
    (bench.harness.measure with CUDA syncs at the loop's events, bench.latency.summarize): p50
    over `repeats` requests, after the timed region."""
    from bench.harness import measure, synchronizer
    from bench.latency import summarize
    from cache.kv import KVCache
    from spec.draft import ModelDraft
    from spec.loop import generate

    def request(watch) -> int:
        cache = KVCache.for_model(target.config, num_blocks=blocks, block_size=BLOCK, dtype=torch.bfloat16, device=device)
        dcache = KVCache.for_model(draft.config, num_blocks=blocks, block_size=BLOCK, dtype=torch.bfloat16,
                                   device=device)
        out, _ = generate(target, cache, ModelDraft(draft, dcache), prompts, NEW_TOKENS, k=K, on_event=watch.mark)
        return sum(len(o) for o in out)

    s = summarize(measure({"spec_draft": request}, warmup=0, repeats=repeats, sync=synchronizer(device), seed=0))
    s = s["spec_draft"]
    p50 = lambda d: d["p50"] if d else None  # noqa: E731
    return {"requests": s["n"], "tokens_per_request": p50(s["tokens"]), "ttft_ms": p50(s["ttft_ms"]),
            "ttft_first_round_ms": p50(s["ttft_first_round_ms"]), "draft_prefill_ms": p50(s["draft_prefill_ms"]),
            "tpot_ms": p50(s["tpot_ms"]), "tpot_first_round_ms": p50(s["tpot_first_round_ms"]),
            "e2e_ms": p50(s["e2e_ms"]),
            "source": "bench.harness.measure + bench.latency.summarize (p50; device synced at each event)"}


REF_SAMPLE_NEW = 4  # generated tokens per reference-arm sample: the first token and three rounds


def reference_request_rate(target, draft, prompt: list[int], w: dict, emitted_per_round: float | None = None) -> dict:
    """One bounded sample of a workload's request through the reference's own stock code path
    (installed unmodified under baseline/_ref): spec.loop.generate with its ModelDraft or
    NGramDraft and cache.kv.KVCache on the host cores, REF_SAMPLE_NEW tokens (prefills, first
    token, then rounds). The loop's own events split the time into the prefill part and the
    rounds; tokens/s of the full request is its token count over the prefill part plus the
    rounds a full request needs (at the sample's mean emitted tokens per round, or
    `emitted_per_round` when given) at the sample's time per round."""
    import math

    from cache.kv import KVCache
    from spec.draft import ModelDraft
    from spec.loop import generate
    from spec.ngram import NGramDraft

    blocks = (w["prompt"] + w["new"] + 2 * w["k"] + 8) // w["block"] + 2
    tc = KVCache.for_model(target.config, num_blocks=blocks, block_size=w["block"], dtype=torch.bfloat16, device="cpu")
    if w["drafter"] == "model":
        dc = KVCache.for_model(draft.config, num_blocks=blocks, block_size=w["block"], dtype=torch.bfloat16,
                               device="cpu")
        drafter = ModelDraft(draft, dc)
    else:
        drafter = NGramDraft(TARGET["vocab_size"], max_n=3)
    ev: dict[str, float] = {}
    t0 = time.perf_counter()
    _, st = generate(target, tc, drafter, [prompt], REF_SAMPLE_NEW, k=w["k"], temperature=w["T"],
                     generator=torch.Generator().manual_seed(0),
                     on_event=lambda name: ev.setdefault(name, time.perf_counter() - t0))
    t_end = time.perf_counter() - t0
    per_round = (t_end - ev["draft_prefilled"]) / max(1, st.rounds)
    emitted = emitted_per_round or max(1.0, (REF_SAMPLE_NEW - 1) / max(1, st.rounds))
    rounds_full = math.ceil((w["new"] - 1) / emitted)
    total = ev["draft_prefilled"] + rounds_full * per_round
    return {"value": w["new"] / total, "prefill_s": ev["draft_prefilled"], "round_s": per_round,
            "rounds_full": rounds_full, "sample_rounds": st.rounds}


def port_request_rate(target, draft, prompt: list[int], engine_rounds: int | None, max_rounds: int = 2) -> dict:
    """The CPU oracle (the numpy restatement of the reference path under oracle/) on this host:
    target and draft prefill, first token and `max_rounds` rounds of config 2, extrapolated to
    the full 256-token request with the given round count (the same greedy algorithm makes the
    same number of rounds), or with the sample's own acceptance."""
    from oracle import forward as ofw
    from oracle import loop as oloop

    prec = ofw.Precision("bf16")
    tw = ofw.weights_from_model(target)
    dw = ofw.weights_from_model(draft)
    drafter = oloop.ModelDraft(dw, prec, num_blocks=64, block_size=BLOCK)
    _, st = oloop.generate(tw, prec, drafter, [prompt], NEW_TOKENS, K, num_blocks=64, block_size=BLOCK,
                           max_rounds=max_rounds)
    per_round = st["seconds_rounds"] / max(1, st["rounds"])
    if engine_rounds is None:
        emitted = max(1.0, sum(st["emitted_per_round"]) / max(1, len(st["emitted_per_round"])))
        engine_rounds = int(np.ceil((NEW_TOKENS - 1) / emitted))
    total = st["seconds_prefill"] + per_round * engine_rounds
    return {"value": NEW_TOKENS / total, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": (f"CPU oracle (numpy, bf16 rounding) on config 2 at B=1: prefill of the {PROMPT_LEN}-token "
                       f"prompt on target and draft + first token ({st['seconds_prefill']:.2f} s) and "
                       f"{st['rounds']} rounds ({per_round:.3f} s each), extrapolated to {engine_rounds} rounds "
                       f"for {NEW_TOKENS} tokens")}


def reference_arm(args, w: dict, config: dict) -> dict:
    """`--impl reference`: the workload's request through the reference's own CPU code
    (baseline/_ref) on all host cores, K bounded samples after at most one warm-up sample; for
    config 2 the numpy port is timed once beside it. Falls back to the port alone when the
    reference is not installed (config 2 only)."""
    torch.set_num_threads(os.cpu_count() or 1)
    target = make_model(TARGET, 0, "cpu")
    draft = make_model(DRAFT, 1, "cpu") if w["drafter"] == "model" else None
    prompt = workload_prompts(w, 0, 1)[0]
    if REF_INSTALL.is_dir():
        for _ in range(min(args.warmup, 1)):
            reference_request_rate(target, draft, prompt, w)
        samples = [reference_request_rate(target, draft, prompt, w) for _ in range(max(1, args.steps))]
        v = statistics.median(s["value"] for s in samples)
        mid = sorted(samples, key=lambda s: s["value"])[len(samples) // 2]
        cb = {"value": v, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "reference",
              "sample": (f"the reference's spec.loop.generate (installed unmodified under baseline/_ref) on one "
                         f"{w['name']} request on the host cores, {len(samples)} samples of {REF_SAMPLE_NEW} tokens: "
                         f"prefill + first token {mid['prefill_s']:.2f} s, {mid['round_s']:.3f} s per round, "
                         f"extrapolated to {mid['rounds_full']} rounds for {w['new']} tokens (median)")}
        port = None
        if w["name"] == "config2" and not args.no_cpu_baseline:
            try:
                port = port_request_rate(target, draft, prompt, engine_rounds=mid["rounds_full"])
                port["vs_reference"] = port["value"] / v
            except Exception as e:  # noqa: BLE001
                port = {"value": None, "sample": f"failed: {e}"}
        cb["port"] = port
    else:
        if w["name"] != "config2":
            return {"impl": "reference", "unavailable": "the reference is not installed under baseline/_ref"}
        cb = port_request_rate(target, draft, prompt, engine_rounds=None)
        v = cb["value"]
    return {"impl": "reference", "metric": w["metric"], "value": v, "unit": "tokens/s", "n_gpus": 0,
            "steps": args.steps, "warmup": min(args.warmup, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config, "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def cpu_baseline_subprocess(config_id: int, steps: int = 3) -> dict | None:
    """The reference arm's measurement, run as a separate process (its packages cannot share
    this process with the engine's): its cpu_baseline object."""
    cmd = [sys.executable, str(Path(__file__).resolve()), "--impl", "reference", "--config", str(config_id), "--steps",
           str(steps), "--warmup", "1", "--no-cpu-baseline"]
    try:
        res = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
        lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
        return json.loads(lines[-1])["cpu_baseline"] if lines else {"value": None, "sample": res.stderr[-500:]}
    except Exception as e:  # noqa: BLE001
        return {"value": None, "sample": f"failed: {e}"}


def time_requests(run, reps: int) -> dict:
    """`run()` generates one batch and returns (tokens, SpecStats or None); device time with
    CUDA events around `reps` calls after one warm-up call."""
    run()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    tokens = rounds = accepted = drafted = 0
    for _ in range(reps):
        n, st = run()
        tokens += n
        if st is not None:
            rounds, accepted, drafted = rounds + st.rounds, accepted + st.accepted, drafted + st.drafted
    ev1.record()
    ev1.synchronize()
    s = ev0.elapsed_time(ev1) / 1e3
    out = {"value": tokens / s, "unit": "tokens/s", "ms_per_request": s * 1e3 / reps, "requests": reps}
    if drafted:
        out.update({"acceptance": accepted / drafted, "rounds_per_request": rounds / reps})
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["engine", "reference"], default="engine")
    ap.add_argument("--config", type=int, choices=sorted(WORKLOADS), default=2,
                    help="BASELINE workload: 2 (default; 1.7B + 135M draft, B=1), 4 (32 requests per GPU, k=8, "
                         "T=0.8) or 5 (8k-token prompts, n-gram drafter)")
    ap.add_argument("--batch", type=int, default=0,
                    help="requests per GPU, overriding the workload's (e.g. --config 2 --batch 64 for the metric's "
                         "@B64 point)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="config 2: skip the accept microbench, latency, plain-decode and noisy-draft lines")
    ap.add_argument("--layers", type=int, default=0,
                    help="with --only: build the models with this many layers (smaller profiling runs)")
    ap.add_argument("--draft-tokens", type=int, default=1,
                    help="with --only draft: new tokens per draft forward (2 = a round's first step)")
    ap.add_argument("--trace", action="store_true",
                    help="with --only verify/draft: per-launch timings from globaltimer stamps")
    ap.add_argument("--only", choices=["verify", "accept", "draft"],
                    help="time one piece alone (for profiling): the verify forward, the accept kernel or one "
                         "draft-model forward step")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    w = dict(WORKLOADS[args.config])
    if args.batch > 0 and args.batch != w["B"]:
        w["B"] = args.batch
        w["metric"] = w["metric"].replace("@B1 ", f"@B{args.batch} ").replace("@B32 ", f"@B{args.batch} ")
        w["workload"] = w["workload"].replace("B=1 per GPU", f"B={args.batch} per GPU").replace(
            "32 requests per GPU", f"{args.batch} requests per GPU")
    B = w["B"]
    config = {"workload": w["workload"], "global_batch": B * world, "seq_len": w["prompt"] + w["new"],
              "parallelism": f"requests sharded x{world}",
              "l2": "weights 3.4 GB >> 126 MB L2 (no flush needed); accept microbench flushes L2 between launches (write 256 MB, then read 256 MB)"}

    if args.impl == "reference":
        if rank != 0:
            return
        print(json.dumps(reference_arm(args, w, config)))
        return

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.only:
        from cache.kv import KVCache

        pk = peaks()
        if args.only == "accept":
            r = time_accept(device, reps=max(1, args.steps))
        elif args.only == "verify":
            spec = dict(TARGET, num_hidden_layers=args.layers or TARGET["num_hidden_layers"])
            r = time_verify_step(make_model(spec, 0, device), KVCache, device, w["prompt"] + w["new"] // 2,
                                 reps=max(1, args.steps), trace=args.trace, B=B, k=w["k"], block=w["block"])
        else:
            spec = dict(DRAFT, num_hidden_layers=args.layers or DRAFT["num_hidden_layers"])
            r = time_draft_step(make_model(spec, 1, device), KVCache, device, PROMPT_LEN + NEW_TOKENS // 2,
                                reps=max(1, args.steps), trace=args.trace, tokens=args.draft_tokens)
        r["gbs"] = r["bytes"] / (r["us"] * 1e-6) / 1e9
        r["frac"] = r["gbs"] / pk["hbm_gbs"]
        print(json.dumps({"only": args.only, **r}))
        return
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    from cache.kv import KVCache
    from spec.draft import ModelDraft
    from spec.loop import generate
    from spec.ngram import NGramDraft

    from specb200.shard import gather_results, shard_range

    target = make_model(TARGET, 0, device)
    draft = make_model(DRAFT, 1, device) if w["drafter"] == "model" else None
    # the box's requests are sharded as contiguous ranges, B per rank
    lo, hi = shard_range(B * world, rank, world)
    prompts = workload_prompts(w, lo, hi - lo)
    per_req = -(-(w["prompt"] + w["new"] + 2 * w["k"] + 8) // w["block"]) + 1
    blocks = len(prompts) * per_req + 2

    def step():
        cache = KVCache.for_model(target.config, num_blocks=blocks, block_size=w["block"], dtype=torch.bfloat16,
                                  device=device)
        if w["drafter"] == "model":
            dcache = KVCache.for_model(draft.config, num_blocks=blocks, block_size=w["block"], dtype=torch.bfloat16,
                                       device=device)
            drafter = ModelDraft(draft, dcache)
        else:
            drafter = NGramDraft(TARGET["vocab_size"], max_n=3)
        gen = torch.Generator().manual_seed(1234)
        return generate(target, cache, drafter, prompts, w["new"], k=w["k"], temperature=w["T"], generator=gen)

    for _ in range(args.warmup):
        out, stats = step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clocks:
        torch.cuda.synchronize()
        ev0.record()
        w0 = time.perf_counter()
        tokens = rounds = accepted = drafted = 0
        for _ in range(args.steps):
            out, stats = step()
            tokens += sum(len(o) for o in out)
            rounds += stats.rounds
            accepted += stats.accepted
            drafted += stats.drafted
        ev1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - w0
    dev_s = ev0.elapsed_time(ev1) / 1e3
    per_rank = {"device_s": dev_s, "tokens": tokens}
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([dev_s, wall, float(tokens)], device=device, dtype=torch.float64)
        every = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(every, t)
        dev_s = max(float(x[0]) for x in every)
        wall = max(float(x[1]) for x in every)
        tokens_all = sum(float(x[2]) for x in every)
        per_rank = {"device_s": [round(float(x[0]), 4) for x in every], "tokens": [int(x[2]) for x in every]}
        # the last step's outputs and statistics of every request (kilobytes), over NCCL
        # after the timed region
        out, stats = gather_results(out, stats, device=device)
    else:
        tokens_all = float(tokens)
    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    pk = peaks()
    vstep = time_verify_step(target, KVCache, device, w["prompt"] + w["new"] // 2, B=len(prompts), k=w["k"],
                             block=w["block"])
    achieved = vstep["bytes"] / (vstep["us"] * 1e-6) / 1e9
    alpha = accepted / max(1, drafted)
    from specb200.engine import engine_for

    te = engine_for(target)
    nb = len(prompts)
    if w["drafter"] == "model":
        de = engine_for(draft)
        # per round: k x (draft forward + sampler + token scatter), verify ids, verify forward,
        # accept, commit; per step: target and draft prefill forwards and the first-token sampler
        per_round = w["k"] * (de.launches(nb, 2) + 2) + 1 + te.launches(nb, w["k"] + 1) + 2
        per_step = te.launches(nb, w["prompt"]) + de.launches(nb, w["prompt"]) + 1
    else:
        per_round = 1 + 1 + te.launches(nb, w["k"] + 1) + 2  # n-gram, verify ids, forward, accept, commit
        per_step = te.launches(nb, w["prompt"]) + 1
    launches = args.steps * per_step + rounds * per_round
    value = tokens_all / dev_s
    line = {
        "metric": w["metric"], "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_s * 1e3 / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, seeded synthetic prompts)",
        "config": config,
        "e2e": {"value": tokens_all / wall, "unit": "tokens/s",
                "h2d_bytes_per_step": w["prompt"] * 8 * B * world, "d2h_bytes_per_step": w["new"] * 8 * B * world},
        "roofline": {"bound": "hbm", "kernel": f"verify step ({len(prompts)} x {w['k'] + 1}-token target forward, "
                                               "CUDA graph)",
                     "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "traffic": vstep["bytes"] * VERIFY_TRAFFIC_RATIO["layers"],
                     "traffic_source": "ncu capture of the 6-layer B=1 verify, scaled by algorithmic bytes",
                     "peak_source": pk["source"], "verify_step_us": vstep["us"],
                     "algorithmic_bytes": vstep["bytes"], "context_tokens": vstep["context"]},
        "acceptance": alpha, "rounds_per_step": rounds / args.steps,
        "per_rank": per_rank,
        "gpu_launches": launches,
        "clocks": clocks.summary(),
    }
    if w["name"] == "config2" and not args.no_extras:
        from baselines import cached_autoregressive
        from spec.draft import NoisyDraft

        acc = time_accept(device)
        acc_gbs = acc["bytes"] / (acc["us"] * 1e-6) / 1e9
        line["accept"] = {"us": acc["us"], "achieved": acc_gbs, "frac": acc_gbs / pk["hbm_gbs"], "unit": "GB/s",
                          "algorithmic_bytes": acc["bytes"], "config": "B=64, k=4, V=49152 fp32 logits, T=1"}
        try:
            line["latency"] = request_latency(target, draft, prompts, device, blocks)
        except Exception as e:  # noqa: BLE001  (the throughput line must still be printed)
            line["latency"] = {"error": f"{type(e).__name__}: {e}"}

        def plain():
            cache = KVCache.for_model(target.config, num_blocks=blocks, block_size=w["block"], dtype=torch.bfloat16,
                                      device=device)
            return len(cached_autoregressive.generate(target, cache, prompts[0], w["new"])), None

        def noisy():
            cache = KVCache.for_model(target.config, num_blocks=blocks, block_size=w["block"], dtype=torch.bfloat16,
                                      device=device)
            dcache = KVCache.for_model(target.config, num_blocks=blocks, block_size=w["block"], dtype=torch.bfloat16,
                                       device=device)
            o, st = generate(target, cache, NoisyDraft(target, dcache, sigma=NOISY_SIGMA, seed=0), prompts[:1],
                             w["new"], k=w["k"])
            return len(o[0]), st

        line["plain"] = time_requests(plain, 3)
        line["plain"]["source"] = "baselines.cached_autoregressive.generate on the engine (one graph replay per token)"
        line["spec_vs_plain"] = value / world / line["plain"]["value"]
        nz = time_requests(noisy, 3)
        nz.update({"sigma": NOISY_SIGMA, "drafter": "spec.draft.NoisyDraft: the target itself + N(0, sigma^2) on "
                                                   "its final logits (config 2's second variant)"})
        line["variants"] = {"config2b_noisy_draft": nz}
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline_subprocess(args.config, steps=3 if args.config == 2 else 1)
    print(json.dumps(line))
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
