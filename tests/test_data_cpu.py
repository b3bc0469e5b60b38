"""Training data on CPU: the byte-offset JSONL index (blank lines, missing
final newline, rank striding), row encoding for pre-tokenized / chat / text
rows with a stand-in tokenizer, skipping of invalid rows, the prefetch
thread, and a trainer run reading a chat JSONL through the index."""
import json

import pytest
import torch

from d3d_b200.train.data import IndexedExamples, JsonlIndex, Prefetcher, RowLimits, encode_row


class ToyTokenizer:
    """Character-level stand-in with a chat template: each turn renders as
    ``<role>:content|`` and the generation prompt as ``<assistant>:``."""
    eos_token_id = 3

    def encode(self, text, add_special_tokens=False):
        return [10 + (ord(c) % 200) for c in text]

    def apply_chat_template(self, msgs, tokenize=False, add_generation_prompt=False, enable_thinking=False):
        text = "".join(f"<{m['role']}>:{m['content']}|" for m in msgs)
        if add_generation_prompt:
            text += "<assistant>:"
        return self.encode(text) if tokenize else text


def _write(path, lines, trailing_newline=True):
    path.write_text("\n".join(lines) + ("\n" if trailing_newline else ""))


def test_index_offsets_blank_lines_and_rank_striding(tmp_path):
    rows = [json.dumps({"prompt_ids": [i + 1], "response_ids": [5, 6, 7]}) for i in range(7)]
    lines = [rows[0], "", rows[1], "   ", rows[2], rows[3], "", rows[4], rows[5], rows[6]]
    p = tmp_path / "d.jsonl"
    _write(p, lines, trailing_newline=False)
    full = JsonlIndex(str(p))
    assert len(full) == 7 and [full.row(i)["prompt_ids"][0] for i in range(7)] == list(range(1, 8))
    r1 = JsonlIndex(str(p), rank=1, world=3)
    assert [r1.global_row(i) for i in range(len(r1))] == [1, 4]
    assert [r1.row(i)["prompt_ids"][0] for i in range(len(r1))] == [2, 5]
    capped = JsonlIndex(str(p), max_rows=4)
    assert len(capped) == 4


def test_encode_row_formats_and_skips():
    tok = ToyTokenizer()
    assert encode_row({"prompt_ids": [1, 2], "response_ids": [3, 4]}).response_ids == [3, 4]
    chat = {"conversations": [{"from": "human", "value": "hi"}, {"from": "gpt", "value": "yo!"}]}
    ex = encode_row(chat, tok)
    full = tok.apply_chat_template([{"role": "user", "content": "hi"}, {"role": "assistant", "content": "yo!"}],
                                   tokenize=True)
    assert ex.prompt_ids + ex.response_ids == full
    assert ex.prompt_ids == tok.apply_chat_template([{"role": "user", "content": "hi"}], tokenize=True,
                                                    add_generation_prompt=True)
    assert encode_row({"prompt": "ab", "response": "cde"}, tok).response_ids == tok.encode("cde")
    # skipped: failed status, one-token response, no assistant turn, too long
    assert encode_row({"status": "error", "prompt_ids": [1], "response_ids": [2, 3]}) is None
    assert encode_row({"prompt_ids": [1], "response_ids": [2]}) is None
    assert encode_row({"messages": [{"role": "user", "content": "x"}]}, tok) is None
    assert encode_row({"prompt_ids": [1] * 10, "response_ids": [2, 3]}, limits=RowLimits(max_prompt_len=5)) is None


def test_indexed_examples_take_wraps_and_counts_skips(tmp_path):
    lines = [json.dumps({"prompt_ids": [i + 1], "response_ids": [5, 6] if i % 3 else [5]}) for i in range(6)]
    p = tmp_path / "d.jsonl"
    _write(p, lines)
    src = IndexedExamples(str(p), 0, 1)
    got, cur = src.take(0, 3)
    assert [e.prompt_ids[0] for e in got] == [2, 3, 5] and cur == 5 and src.skipped == 2
    got, cur = src.take(cur, 2)       # wraps around the end of the file
    assert [e.prompt_ids[0] for e in got] == [6, 2]


def test_prefetcher_order_and_errors():
    pf = Prefetcher(lambda s: s * s, 2, 6, depth=2)
    assert [pf.get() for _ in range(4)] == [(2, 4), (3, 9), (4, 16), (5, 25)]
    with pytest.raises(StopIteration):
        pf.get()

    def boom(s):
        if s == 1:
            raise RuntimeError("bad row")
        return s
    pf = Prefetcher(boom, 0, 3)
    assert pf.get() == (0, 0)
    with pytest.raises(RuntimeError, match="bad row"):
        pf.get()


def test_trainer_reads_chat_jsonl(tmp_path, monkeypatch):
    from d3d_b200.train import trainer
    from d3d_b200.train.args import parser
    import transformers
    monkeypatch.setattr(transformers.AutoTokenizer, "from_pretrained", staticmethod(lambda *a, **k: ToyTokenizer()))
    rows = []
    for i in range(6):
        rows.append(json.dumps({"messages": [{"role": "user", "content": f"question {i} " * 3},
                                             {"role": "assistant", "content": f"answer number {i} " * 4}]}))
    p = tmp_path / "chat.jsonl"
    _write(p, rows)
    a = parser().parse_args(["--draft-model", "tiny-drafter", "--output-dir", str(tmp_path / "out"),
                             "--data-path", str(p), "--tokenizer", "toy", "--batch-size", "2",
                             "--parallel-anchors-per-example", "3", "--max-steps", "3", "--block-size", "8",
                             "--vocab-chunk", "256", "--objective", "ce", "--device", "cpu", "--dtype", "fp32"])
    r = trainer.train(a)
    assert len(r["log"]) == 3 and all(torch.isfinite(torch.tensor(x["loss"])) for x in r["log"])
    assert all(x["tokens"] > 0 for x in r["log"])
