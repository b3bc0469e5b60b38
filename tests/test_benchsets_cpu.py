"""Evaluation sets: both local cache layouts, gold answers, exact-answer
scoring, and the CLI path that renders questions with the chat template and
reports accuracy."""
import argparse
import json

import pytest

from d3d_b200.utils.benchsets import SETS, canonical, extract_answer, last_boxed, load_set, score


def test_answer_extraction_and_canonical_form():
    assert last_boxed(r"so \boxed{\frac{1}{2}} and later \boxed{42}") == "42"
    assert last_boxed(r"x = \boxed{\frac{a}{b^{2}}}") == r"\frac{a}{b^{2}}"
    assert last_boxed(r"\boxed{unclosed") is None and last_boxed("none") is None
    assert extract_answer(r"The answer is $\boxed{$1,234$}$.") == "1,234"
    assert extract_answer("we get 12 then 3,400 apples") == "3400"
    assert extract_answer("no digits") is None
    assert canonical("1,234.") == "1234" and canonical(" 3.0 ") == "3" and canonical("2.5") == "2.5"
    assert canonical(r"\!7") == "7" and canonical("(3, 2)") == "(32)" and canonical("inf") == "inf"
    assert score("gsm8k", r"... \boxed{1,234}", "1234") == ("1,234", True)
    assert score("gsm8k", "... 17", "18") == ("17", False)
    assert score("math500", "x", None) == (None, None)
    assert score("humaneval", "def f(): pass", "x") == (None, None)
    assert sorted(SETS) == ["aime25", "gsm8k", "humaneval", "livecodebench-v6", "math500", "mbpp", "mt-bench"]


def test_reference_cache_layout(tmp_path):
    data, ans = tmp_path / "data", tmp_path / "ans"
    data.mkdir()
    ans.mkdir()
    (data / "gsm8k.jsonl").write_text("\n".join(json.dumps({"turns": [f"Q{i}?"]}) for i in range(3)) + "\n")
    (ans / "gsm8k.jsonl").write_text("\n".join(json.dumps({"answer": f"steps\n#### {i},000"}) for i in range(3)))
    exs, meta = load_set("gsm8k", data_dir=data, answer_dir=ans)
    assert [e.question for e in exs] == ["Q0?", "Q1?", "Q2?"]
    assert [e.gold for e in exs] == ["0000", "1000", "2000"]
    assert meta["samples"] == 3 and meta["scored"] and len(meta["sha256"]) == 64
    (ans / "gsm8k.jsonl").write_text(json.dumps({"answer": "1"}) + "\n")
    with pytest.raises(ValueError, match="rows"):
        load_set("gsm8k", data_dir=data, answer_dir=ans)


def test_upstream_row_layout_and_errors(tmp_path):
    rows = [{"problem": "What is 1+1?", "answer": " 2 "}, {"problem": "And 2+2?", "answer": "4"}]
    (tmp_path / "math500.jsonl").write_text("\n".join(json.dumps(r) for r in rows))
    exs, _ = load_set("math500", max_samples=1, data_dir=tmp_path, answer_dir=tmp_path / "none")
    assert len(exs) == 1 and exs[0].gold == "2"
    assert exs[0].question.startswith("What is 1+1?") and exs[0].question.endswith("\\boxed{}.")
    (tmp_path / "humaneval.jsonl").write_text(json.dumps({"prompt": "def f(x):\n"}) + "\n")
    he, meta = load_set("humaneval", data_dir=tmp_path, answer_dir=tmp_path / "none")
    assert he[0].question.startswith("Write a solution") and "```python\ndef f(x):" in he[0].question
    assert he[0].gold is None and not meta["scored"]
    with pytest.raises(KeyError):
        load_set("nope", data_dir=tmp_path)
    with pytest.raises(FileNotFoundError, match="openai/gsm8k"):
        load_set("gsm8k", data_dir=tmp_path / "missing")


class _ByteTokenizer:
    """Byte-level stand-in for an HF tokenizer (chat template included)."""
    eos_token_id = 0

    def apply_chat_template(self, msgs, tokenize=False, add_generation_prompt=True, enable_thinking=False):
        return "<u>" + msgs[-1]["content"] + "<a>" + ("<think>" if enable_thinking else "")

    def encode(self, text, add_special_tokens=True):
        return list(text.encode())

    def decode(self, ids, skip_special_tokens=False):
        return bytes(ids).decode(errors="replace")


def test_cli_prompts_and_accuracy(tmp_path, monkeypatch):
    import transformers
    from d3d_b200.cli.common import load_prompts, score_outputs
    monkeypatch.setattr(transformers.AutoTokenizer, "from_pretrained", staticmethod(lambda *a, **k: _ByteTokenizer()))
    monkeypatch.setenv("D3D_DATA_CACHE", str(tmp_path))
    monkeypatch.setenv("D3D_ANSWER_CACHE", str(tmp_path / "ans"))
    rows = [{"question": "2+3?", "answer": "#### 5"}, {"question": "2*3?", "answer": "#### 6"}]
    (tmp_path / "gsm8k.jsonl").write_text("\n".join(json.dumps(r) for r in rows))
    a = argparse.Namespace(dataset="gsm8k", tokenizer="fake", max_samples=8, enable_thinking=False,
                           target="tiny-target", prompt_min=1, prompt_max=2, seed=0)
    prompts = load_prompts(a)
    assert bytes(prompts[0]).decode().startswith("<u>2+3?")
    outs = [list(r"so \boxed{5}".encode()), list(b"it is 7")]
    acc = score_outputs(a, outs)
    assert acc["scored"] == 2 and acc["correct"] == 1 and acc["accuracy"] == 0.5
    assert [r["correct"] for r in acc["rows"]] == [True, False]
