"""The offline benchmark module on CPU with the tiny model: random-length prompts, and a
WildChat-style parquet shard whose first user turns are filtered by language and flags."""

import json

import pytest

from minisgl.models.synthetic import make_checkpoint


def test_random_prompts(tmp_path, capsys):
    from minisgl.benchmark.offline import main

    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"))
    res = main(["--model", path, "--device", "cpu", "--dtype", "float32", "--dummy-weight", "--num-seqs", "5",
                "--input-range", "5,30", "--output-range", "2,7", "--max-running-requests", "4"])
    assert res["requests"] == 5 and res["output_tokens"] == res["output_budget"] > 0
    line = [l for l in capsys.readouterr().out.splitlines() if l.startswith("{")][-1]
    assert json.loads(line)["output_tokens"] == res["output_tokens"]


@pytest.mark.parametrize("fmt", ["parquet", "jsonl"])
def test_wildchat_style_dataset(tmp_path, fmt):
    from minisgl.benchmark.offline import iter_dataset_texts, main

    convs = [
        [{"role": "user", "content": "hello there", "language": "English", "redacted": False, "toxic": False},
         {"role": "assistant", "content": "hi", "language": "English", "redacted": False, "toxic": False}],
        [{"role": "user", "content": "bonjour", "language": "French", "redacted": False, "toxic": False}],
        [{"role": "user", "content": "bad words", "language": "English", "redacted": False, "toxic": True}],
        [{"role": "user", "content": "ni hao", "language": "Chinese", "redacted": False, "toxic": False}],
        [],
    ]
    f = tmp_path / f"shard.{fmt}"
    if fmt == "parquet":
        import pyarrow as pa
        import pyarrow.parquet as pq

        pq.write_table(pa.table({"conversation": convs}), str(f))
    else:
        f.write_text("\n".join(json.dumps({"conversation": c}) for c in convs) + "\n" + json.dumps({"prompt": "plain"}))
    want = ["hello there", "ni hao"] + (["plain"] if fmt == "jsonl" else [])
    assert list(iter_dataset_texts(str(f))) == want
    path = make_checkpoint("tiny-qwen3", str(tmp_path / "m"))
    res = main(["--model", path, "--device", "cpu", "--dtype", "float32", "--dummy-weight", "--dataset", str(f),
                "--max-output", "4", "--ignore-eos", "--temperature", "0.6"])
    assert res["requests"] == len(want) and res["output_tokens"] == 4 * len(want)
