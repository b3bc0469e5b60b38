"""Evaluation sets by name, with their questions, gold answers and scoring.

The reference reports its results on seven public sets
(``common/data.py:73-136``: GSM8K, MATH-500, AIME 2025, HumanEval, MBPP,
MT-Bench, LiveCodeBench v6) and scores the math sets by exact final answer
(``common/data.py:202-236``).  Nothing is downloaded here: a set is read from
a local cache directory, in either of two layouts per set ``NAME``:

* ``NAME.jsonl`` whose rows carry ``turns`` (the question is the first turn),
  with the gold answers, if any, as aligned rows of ``NAME.jsonl`` in a
  separate answer directory -- the reference's own cache layout, so existing
  caches are reused as they are;
* ``NAME.jsonl`` whose rows are the upstream dataset's rows (``question`` /
  ``answer`` for GSM8K, ``problem`` / ``answer`` for MATH-500, ...): the
  question and gold answer are derived from the row's fields.

The default directories are ``$D3D_DATA_CACHE`` and ``$D3D_ANSWER_CACHE``
(the reference's variable names), else ``data_cache`` / ``answer_cache`` in
the working directory.

Scoring extracts the last ``\\boxed{...}`` of the output (braces matched),
else its last number, and compares it with the gold answer after the same
canonicalisation on both sides (spacing, commas, a trailing period, ``\\!``
removed; integral numbers written without a decimal part).
"""
from __future__ import annotations

import hashlib
import json
import math
import os
import re
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable, Dict, List, Optional, Tuple

REASON = "\nPlease reason step by step, and put your final answer within \\boxed{}."
CODE_LEAD = "Write a solution to the following problem and make sure that it passes the tests:"


@dataclass(frozen=True)
class BenchSet:
    name: str
    upstream: Tuple[str, Optional[str], str]      # hub id, subset, split the rows come from
    question: Callable[[Dict[str, Any]], str]
    gold: Optional[Callable[[Dict[str, Any]], Optional[str]]]
    scored: bool                                  # exact-final-answer scoring applies


def _given(row: Dict[str, Any]) -> Optional[str]:
    p = row.get("prompt")
    if isinstance(p, list):
        p = p[0] if p else None
    return p if isinstance(p, str) and p else None


def _math_question(field: str) -> Callable[[Dict[str, Any]], str]:
    return lambda row: _given(row) or str(row[field]) + REASON


def _gsm8k_gold(row: Dict[str, Any]) -> Optional[str]:
    ans = row.get("answer")
    if ans is None:
        return None
    return str(ans).rsplit("####", 1)[-1].strip().replace(",", "")


def _plain_gold(row: Dict[str, Any]) -> Optional[str]:
    ans = row.get("answer")
    return None if ans is None else str(ans).strip()


def _humaneval_question(row: Dict[str, Any]) -> str:
    p = _given(row) or ""
    return p if p.startswith(CODE_LEAD.split(" and ")[0]) else f"{CODE_LEAD}\n```python\n{p}\n```"


def _lcb_question(row: Dict[str, Any]) -> str:
    p = _given(row)
    if p:
        return p
    parts = [CODE_LEAD]
    for key in ("question_title", "question_content"):
        v = str(row.get(key) or "").replace("\r\n", "\n").strip()
        if v:
            parts.append(v)
    if row.get("starter_code"):
        parts.append("Starter code:\n```python\n" + str(row["starter_code"]) + "\n```")
    return "\n\n".join(parts)


SETS: Dict[str, BenchSet] = {s.name: s for s in (
    BenchSet("gsm8k", ("openai/gsm8k", "main", "test"), _math_question("question"), _gsm8k_gold, True),
    BenchSet("math500", ("HuggingFaceH4/MATH-500", None, "test"), _math_question("problem"), _plain_gold, True),
    BenchSet("aime25", ("MathArena/aime_2025", None, "train"), _math_question("problem"), _plain_gold, True),
    BenchSet("humaneval", ("openai/openai_humaneval", None, "test"), _humaneval_question, None, False),
    BenchSet("mbpp", ("google-research-datasets/mbpp", "sanitized", "test"),
             lambda r: _given(r) or str(r["text"]), None, False),
    BenchSet("mt-bench", ("HuggingFaceH4/mt_bench_prompts", None, "train"), lambda r: _given(r) or "", None, False),
    BenchSet("livecodebench-v6", ("livecodebench/code_generation_lite", None, "test"), _lcb_question, None, False),
)}


def cache_dirs() -> Tuple[Path, Path]:
    return (Path(os.environ.get("D3D_DATA_CACHE", "data_cache")),
            Path(os.environ.get("D3D_ANSWER_CACHE", "answer_cache")))


def _jsonl(path: Path) -> List[Dict[str, Any]]:
    return [json.loads(line) for line in path.read_text().splitlines() if line.strip()]


@dataclass
class Example:
    dataset: str
    index: int
    question: str
    gold: Optional[str]


def load_set(name: str, max_samples: Optional[int] = None, data_dir: Optional[Path] = None,
             answer_dir: Optional[Path] = None) -> Tuple[List[Example], Dict[str, Any]]:
    """The examples of set ``name`` from the local cache and a description of
    what was read (source file, sample count, SHA-256 of the examples)."""
    if name not in SETS:
        raise KeyError(f"unknown evaluation set {name!r}; known: {', '.join(sorted(SETS))}")
    spec = SETS[name]
    ddir, adir = cache_dirs()
    ddir, adir = Path(data_dir or ddir), Path(answer_dir or adir)
    src = ddir / f"{name}.jsonl"
    if not src.is_file():
        raise FileNotFoundError(f"no local cache for {name}: {src} (no network here; upstream rows are "
                                f"{spec.upstream[0]} {spec.upstream[1] or ''} {spec.upstream[2]})")
    rows = _jsonl(src)
    ans_path = adir / f"{name}.jsonl"
    answers = _jsonl(ans_path) if ans_path.is_file() else None
    if answers is not None and len(answers) != len(rows):
        raise ValueError(f"{src} has {len(rows)} rows but {ans_path} has {len(answers)}")
    out: List[Example] = []
    for i, row in enumerate(rows):
        turns = row.get("turns")
        if turns is not None:
            if not turns:
                raise ValueError(f"{src} row {i} has no turns")
            q = str(turns[0])
            extra = answers[i] if answers is not None else {}
        else:
            q = spec.question(row)
            extra = dict(row)
            if answers is not None:
                extra.update(answers[i])
        gold = None
        if spec.gold is not None:
            gold = extra.get("gold") if extra.get("gold") is not None else spec.gold(extra)
        out.append(Example(name, i, q, None if gold is None else str(gold)))
        if max_samples and len(out) >= max_samples:
            break
    digest = hashlib.sha256(json.dumps([(e.question, e.gold) for e in out]).encode()).hexdigest()
    return out, {"dataset": name, "source": str(src), "answers": str(ans_path) if answers is not None else None,
                 "samples": len(out), "sha256": digest, "scored": spec.scored}


def last_boxed(text: str) -> Optional[str]:
    """Content of the last ``\\boxed{...}`` in ``text`` (nested braces matched)."""
    at = text.rfind("\\boxed")
    if at < 0:
        return None
    start = text.find("{", at)
    if start < 0:
        return None
    depth = 0
    for j in range(start, len(text)):
        c = text[j]
        if c == "{":
            depth += 1
        elif c == "}":
            depth -= 1
            if depth == 0:
                return text[start + 1:j].strip()
    return None


_NUMBER = re.compile(r"-?\d+(?:\.\d+)?")


def extract_answer(text: str) -> Optional[str]:
    """The final answer of an output: its last boxed expression (dollar signs
    dropped), else its last number (thousands separators ignored)."""
    b = last_boxed(text)
    if b is not None:
        return b.replace("$", "").strip()
    nums = _NUMBER.findall(text.replace(",", ""))
    return nums[-1] if nums else None


def canonical(ans: Optional[str]) -> Optional[str]:
    if ans is None:
        return None
    s = ans.strip().rstrip(".")
    for junk in ("\\!", " ", ","):
        s = s.replace(junk, "")
    try:
        v = float(s)
    except (TypeError, ValueError, OverflowError):
        return s
    if not math.isfinite(v):
        return s
    return str(int(v)) if v == int(v) else str(v)


def score(name: str, output_text: str, gold: Optional[str]) -> Tuple[Optional[str], Optional[bool]]:
    """(extracted answer, correct) for a scored set with a gold answer, else
    (None, None)."""
    if not SETS[name].scored or gold is None:
        return None, None
    pred = extract_answer(output_text)
    return pred, pred is not None and canonical(pred) == canonical(gold)
