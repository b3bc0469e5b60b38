"""Target-only AR baseline at several concurrencies, with the reference's
repeat / retest policy and per-attempt records (reference:
``serving/baseline_concurrency.py``).

    python -m d3d_b200.cli.baseline --target qwen3-8b --datasets synthetic \\
        --concurrency 1 4 8 16 --max-new-tokens 512 --repeats 2 --output-root out/baseline

Per dataset and concurrency: one discarded warm-up over the full workload,
then ``--repeats`` timed attempts; when two attempts disagree by more than
``--slow-fraction`` (the slower below that fraction of the faster, or below
that fraction of the median for more attempts) up to ``--max-retests``
extra attempts run after another warm-up.  Every attempt is kept: the
summary reports median and pooled throughput, min, max and the slow
attempts, with no fastest-run selection.  Throughput is output tokens over
wall seconds of admission, prefill, decode and release.  Before timing, the
first two prompts of each dataset are checked against ``transformers``'
greedy decoding of the same checkpoint (unless skipped or the target is a
preset); a differing token must at least be a teacher-forced argmax tie.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import statistics
import subprocess
from datetime import datetime, timezone
from pathlib import Path
from typing import Dict, List

import torch

from ..engine.spec import EOS_DEFAULT, ar_generate
from ..utils.io import write_json
from ..utils.runtime import runtime_metadata
from .common import add_data_args, is_preset, load_fast_weights, load_module, load_prompts


def parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--target", required=True, help="checkpoint directory or preset")
    add_data_args(p)
    p.add_argument("--datasets", nargs="+", default=None, help="prompt sources (names or files, as --dataset)")
    p.add_argument("--concurrency", nargs="+", type=int, default=[1, 4, 8, 16])
    p.add_argument("--max-new-tokens", type=int, default=2048)
    p.add_argument("--warmup-new-tokens", type=int, default=256)
    p.add_argument("--repeats", type=int, default=2)
    p.add_argument("--max-retests", type=int, default=1)
    p.add_argument("--slow-fraction", type=float, default=0.85)
    p.add_argument("--pages", type=int, default=4096)
    p.add_argument("--page-size", type=int, default=16)
    p.add_argument("--ignore-eos", action="store_true")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    p.add_argument("--reference-device", default=None, help="device of the transformers reference (default --device)")
    p.add_argument("--skip-reference-validation", action="store_true")
    p.add_argument("--batch-sizes", type=int, nargs="+", default=None,
                   help="fixed-batch decode-only mode (serving/baseline_ar.py): each batch size decodes "
                        "--max-new-tokens steps with no stop condition, prefill excluded")
    p.add_argument("--run-id", default=datetime.now(timezone.utc).strftime("%Y%m%d_%H%M%S"))
    p.add_argument("--output-root", type=Path, default=Path("results_baseline"))
    return p


def slow_attempts(cells: List[dict], fraction: float) -> List[int]:
    """Attempts below ``fraction`` of the faster of two, or of the median of more."""
    ref = (max(c["tps"] for c in cells) if len(cells) == 2 else statistics.median(c["tps"] for c in cells))
    return [c["attempt"] for c in cells if c["tps"] < fraction * ref]


def telemetry() -> str:
    """One ``nvidia-smi`` sample (temperature, power, SM clock, utilisation,
    memory) of every GPU; empty where the tool is absent."""
    try:
        return subprocess.run(["nvidia-smi", "--query-gpu=uuid,name,temperature.gpu,power.draw,clocks.sm,"
                               "utilization.gpu,memory.used", "--format=csv"], capture_output=True, text=True,
                              check=False, timeout=30).stdout
    except (OSError, subprocess.SubprocessError):
        return ""


def build_target(a, max_seqs: int, max_context: int):
    """The kernel target on a GPU, the PyTorch oracle on the CPU."""
    dev = torch.device(a.device)
    if dev.type == "cuda":
        from ..engine.fast import FastTarget
        return FastTarget(load_fast_weights(a.target, dev, a.seed), pages=a.pages, page_size=a.page_size,
                          max_seqs=max_seqs, max_context=max_context, device=dev)
    from ..engine.backends import TorchTarget
    return TorchTarget(load_module(a.target, dev, a.seed).eval())


def validate_against_hf(target: str, device, cases: List[List[int]], outputs: List[List[int]], n_new: int,
                        eos, ignore_eos: bool) -> List[dict]:
    """``transformers``' greedy continuation of each case; where it differs,
    the teacher-forced logit regret of this framework's tokens (0 everywhere
    means every differing token is an exact argmax tie)."""
    import transformers
    dev = torch.device(device)
    dt = torch.bfloat16 if dev.type == "cuda" else torch.float32
    hf = transformers.AutoModelForCausalLM.from_pretrained(target, dtype=dt).to(dev).eval()
    checks = []
    for i, (ids, out) in enumerate(zip(cases, outputs)):
        x = torch.tensor([ids], device=dev)
        kw = {"min_new_tokens": n_new} if ignore_eos else {"eos_token_id": list(eos)}
        with torch.inference_mode():
            exp = hf.generate(x, attention_mask=torch.ones_like(x), max_new_tokens=n_new, do_sample=False,
                              pad_token_id=0, **kw)[0, len(ids):].tolist()
        chk = {"index": i, "equal": out == exp, "actual": out, "expected": exp}
        if not chk["equal"] and out:
            with torch.inference_mode():
                lg = hf(torch.tensor([ids + out[:-1]], device=dev)).logits[0, len(ids) - 1:].float()
            chosen = torch.tensor(out, device=dev)
            regret = lg.max(-1).values - lg.gather(1, chosen[:, None])[:, 0]
            chk.update(teacher_forced_logit_regret=regret.tolist(), max_logit_regret=float(regret.max()),
                       numerically_consistent=float(regret.max()) == 0.0)
        checks.append(chk)
    del hf
    return checks


def _table(summary: Dict[str, dict]) -> str:
    lines = ["| Concurrency | Median TPS | Pooled TPS | Min TPS | Max TPS | Attempts | Slow attempts |",
             "|---:|---:|---:|---:|---:|---:|---|"]
    for c, s in summary.items():
        lines.append(f"| {c} | {s['median_tps']:.2f} | {s['pooled_tps']:.2f} | {s['min_tps']:.2f} | "
                     f"{s['max_tps']:.2f} | {s['attempts']} | {s['slow_attempts']} |")
    return "\n".join(lines) + "\n"


def _fixed_batch(a, target, sets, dirs, meta) -> dict:
    """Decode-only throughput at fixed batch sizes (prompts reused cyclically
    when a batch is larger than the set)."""
    from ..engine.spec import ar_decode_fixed
    out = {}
    for name, prompts in sets.items():
        payload = {**meta, "mode": "fixed_batch_decode_only", "dataset": name, "cells": []}
        for b in a.batch_sizes:
            batch = [prompts[i % len(prompts)] for i in range(b)]
            ar_decode_fixed(target, batch, min(8, a.max_new_tokens))          # warm-up
            for rep in range(a.repeats):
                r = ar_decode_fixed(target, batch, a.max_new_tokens)
                if hasattr(target, "leak_check"):
                    target.leak_check()
                r.pop("outputs")
                payload["cells"].append({"batch_size": b, "repeat": rep, **r})
                print(f"DECODE {name} B={b} repeat={rep} TPS={r['tps']:.2f}", flush=True)
        payload["status"] = "complete"
        write_json(str(dirs[name] / "benchmark.json"), payload)
        out[name] = payload
    return out


def main(argv=None) -> dict:
    from ..utils.runtime import required_pages
    a = parser().parse_args(argv)
    if (min(a.concurrency + [a.repeats, a.max_new_tokens, a.warmup_new_tokens, a.pages]) < 1
            or (a.max_samples or 0) < 0 or a.max_retests < 0):
        raise SystemExit("invalid numeric parameter")
    if not 0 < a.slow_fraction < 1:
        raise SystemExit("--slow-fraction must be between zero and one")
    sets, dirs = {}, {}
    for name in a.datasets or [a.dataset]:
        a.dataset = name
        prompts = load_prompts(a)
        if not prompts:
            raise ValueError(f"no prompts: {name}")
        need = max(map(len, prompts)) + a.max_new_tokens + 1
        worst = required_pages([len(p) for p in prompts], a.max_new_tokens, min(max(a.concurrency), len(prompts)),
                               a.page_size, 1)
        if worst > a.pages or need > 16384:
            raise ValueError(f"{name}: KV capacity or context limit insufficient (pages needed {worst})")
        tag = Path(name).stem if Path(name).suffix else name
        d = a.output_root / tag / a.run_id
        d.mkdir(parents=True, exist_ok=False)
        sets[name], dirs[name] = prompts, d
        write_json(str(d / "inputs.json"), {"source": name, "prompts": prompts})
    eos = () if a.ignore_eos else EOS_DEFAULT
    max_ctx = max(len(p) for ps in sets.values() for p in ps) + a.max_new_tokens + 64
    target = build_target(a, max(a.concurrency), max_ctx)
    meta = {"config": {k: (str(v) if isinstance(v, Path) else v) for k, v in vars(a).items()
                       if not k.startswith("eval_")},
            "metric": "output tokens / wall seconds of admission, prefill, decode and release",
            "repeat_policy": "all attempts kept; median and pooled throughput over original and retest attempts",
            "slowdown_policy": f"an attempt below {a.slow_fraction} of the faster of two (median of more) "
                               f"triggers up to {a.max_retests} retests", "device": str(a.device),
            "hardware": torch.cuda.get_device_name(0) if torch.cuda.is_available() else "cpu",
            "torch": torch.__version__, "eos_ids": list(eos), "temperature": 0,
            "runtime": runtime_metadata({"target": a.target})}

    def run(prompts, c, n):
        r = ar_generate(target, prompts, n, eos=eos or EOS_DEFAULT, ignore_eos=a.ignore_eos, concurrency=c)
        if hasattr(target, "leak_check"):
            target.leak_check()
        if r["max_active"] > c:
            raise RuntimeError("admission invariant failed")
        return r

    if a.batch_sizes:
        return _fixed_batch(a, target, sets, dirs, meta)
    checks = []
    if not a.skip_reference_validation and not is_preset(a.target):
        for name, prompts in sets.items():
            cases = prompts[:2]
            outs = run(cases, 2, 16)["outputs"]
            for chk in validate_against_hf(a.target, a.reference_device or a.device, cases, outs, 16, EOS_DEFAULT,
                                           a.ignore_eos):
                checks.append({"dataset": name, **chk})
        for d in dirs.values():
            write_json(str(d / "validation.json"), checks)
        if not all(c["equal"] or c.get("numerically_consistent", False) for c in checks):
            raise RuntimeError("transformers greedy validation failed")
    payloads = {}
    try:
        for name, prompts in sets.items():
            d = dirs[name]
            payload = {**meta, "dataset": name, "requests": len(prompts), "cells": [], "status": "running",
                       "validation": "skipped" if not checks else "passed",
                       "input_sha256": hashlib.sha256(json.dumps(prompts).encode()).hexdigest()}
            payloads[name] = payload
            write_json(str(d / "benchmark.json"), payload)
            for c in a.concurrency:
                run(prompts, c, a.warmup_new_tokens)          # discarded warm-up of the whole workload
                cells, retests = [], 0
                for attempt in range(a.repeats + a.max_retests):
                    if attempt >= a.repeats:
                        if attempt == a.repeats:
                            retests = a.max_retests if slow_attempts(cells, a.slow_fraction) else 0
                        if attempt >= a.repeats + retests:
                            break
                        run(prompts, c, a.warmup_new_tokens)
                    before = telemetry()
                    r = run(prompts, c, a.max_new_tokens)
                    r.update(dataset=name, concurrency=c, attempt=attempt, is_retest=attempt >= a.repeats,
                             telemetry_before=before, telemetry_after=telemetry())
                    raw = d / f"c{c}_attempt{attempt}.json"
                    write_json(str(raw), r)
                    cell = {k: v for k, v in r.items() if k not in ("outputs", "decode_batch_sizes", "latency_s",
                                                                     "finish_reasons", "telemetry_before",
                                                                     "telemetry_after")}
                    cell["raw_file"] = raw.name
                    cells.append(cell)
                    payload["cells"].append(cell)
                    write_json(str(d / "benchmark.json"), payload)
                    print(f"RESULT {name} C={c} attempt={attempt} TPS={r['tps']:.2f}", flush=True)
                payload.setdefault("summary", {})[str(c)] = {
                    "median_tps": statistics.median(x["tps"] for x in cells),
                    "pooled_tps": sum(x["output_tokens"] for x in cells) / sum(x["elapsed_s"] for x in cells),
                    "min_tps": min(x["tps"] for x in cells), "max_tps": max(x["tps"] for x in cells),
                    "attempts": len(cells), "slow_attempts": slow_attempts(cells, a.slow_fraction)}
                write_json(str(d / "benchmark.json"), payload)
                (d / "table.md").write_text(_table(payload["summary"]))
            payload["status"] = "complete"
            write_json(str(d / "benchmark.json"), payload)
    except BaseException as exc:
        for name, d in dirs.items():
            p = payloads.get(name, {**meta, "cells": []})
            if p.get("status") != "complete":
                p.update(status="failed", error=repr(exc))
                write_json(str(d / "benchmark.json"), p)
        raise
    return payloads


if __name__ == "__main__":
    main()
