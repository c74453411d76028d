"""Text corpora (jsonl / parquet / txt) prepared into a byte file and trained on (CPU)."""

import json
import os

import numpy as np

from burn_dragon_b200.cli.train import main
from burn_dragon_b200.train.datasets import corpus_bytes, prepare_corpus

CFG = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")


def test_prepare_jsonl_parquet_and_cache(tmp_path):
    import pyarrow as pa
    import pyarrow.parquet as pq

    src = tmp_path / "corpus"
    src.mkdir()
    (src / "a.jsonl").write_text("\n".join(json.dumps({"text": t, "id": i}) for i, t in enumerate(["héllo", "world"])))
    pq.write_table(pa.table({"text": ["third doc"]}), src / "b.parquet")
    out = prepare_corpus(str(src), str(tmp_path / "cache"))
    data = bytes(corpus_bytes(out))
    assert data == "héllo\n\nworld\n\nthird doc".encode()
    man = json.load(open(out[:-4] + ".json"))
    assert man["documents"] == 3 and man["bytes"] == len(data)
    mtime = os.path.getmtime(out)
    assert prepare_corpus(str(src), str(tmp_path / "cache")) == out and os.path.getmtime(out) == mtime


def test_training_on_a_text_corpus(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    src = tmp_path / "c.jsonl"
    rng = np.random.default_rng(0)
    src.write_text("\n".join(json.dumps({"body": "abc " * int(rng.integers(50, 200))}) for _ in range(40)))
    main(["--config", CFG, "--set", 'dataset.type="jsonl"', "--set", f'dataset.path="{src}"',
          "--set", f'dataset.cache_dir="{tmp_path / "cache"}"', "--set", 'dataset.text_field="body"',
          "--set", "training.max_iters=4", "--set", "training.block_size=64", "--run-name", "txt"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert res["final_loss"] is not None and res["final_loss"] < 5.5  # "abc " is far below ln 256


def test_bpe_corpus_uint16_tokens_through_both_loaders(tmp_path):
    import torch

    from burn_dragon_b200.train.data import FileBytes
    from burn_dragon_b200.train.datasets import token_bytes
    from burn_dragon_b200.train.native_data import NativeBytes
    from burn_dragon_b200.utils.tokenizer import BPETokenizer

    texts = ["the cat sat on the mat " * 20, "the dog sat on the log " * 20]
    tok = BPETokenizer().train(texts, 300)
    tp = tmp_path / "tokenizer.json"
    tp.write_text(json.dumps(tok.to_json()))
    src = tmp_path / "c.txt"
    src.write_text(texts[0] + texts[1])
    out = prepare_corpus(str(src), str(tmp_path / "cache"), tokenizer=str(tp))
    assert token_bytes(out) == 2
    ids = np.fromfile(out, dtype="<u2")
    assert ids.max() >= 256 and ids.tolist() == tok.encode(texts[0] + texts[1])
    fb = FileBytes(out, 2, 8, ratio=1.0)
    x, y = fb.next()
    assert int(x.max()) < 300 and torch.equal(x[:, 1:], y[:, :-1])
    nb = NativeBytes("file", 2, 8, path=out, ratio=1.0, token_bytes=2)
    x2, _ = nb.next()
    nb.close()
    # every native window is a run of consecutive ids of the file
    flat = ids.tolist()
    for row in x2.tolist():
        assert any(flat[i:i + 8] == row for i in range(len(flat) - 8))


def test_bpe_run_then_generate_cli(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.cli.generate import main as gen_main
    from burn_dragon_b200.utils.tokenizer import BPETokenizer

    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    texts = ["hello there friend " * 30]
    tok = BPETokenizer().train(texts, 280)
    tp = tmp_path / "tokenizer.json"
    tp.write_text(json.dumps(tok.to_json()))
    src = tmp_path / "c.txt"
    src.write_text(" ".join(f"{texts[0]} {i}" for i in range(40)))
    main(["--config", CFG, "--set", 'dataset.type="text"', "--set", f'dataset.path="{src}"',
          "--set", f'dataset.cache_dir="{tmp_path / "cache"}"', "--set", f'dataset.tokenizer="{tp}"',
          "--set", "model.vocab_size=288", "--set", "training.max_iters=2", "--set", "training.block_size=32",
          "--set", "training.checkpoint_interval_iters=2", "--run-name", "bpe"])
    run_dir = json.loads(capsys.readouterr().out.strip().splitlines()[-1])["run_dir"]
    assert json.load(open(os.path.join(run_dir, "tokenizer.json")))["type"] == "bpe"
    gen_main(["--run", run_dir, "--prompt", "hello there", "--max-tokens", "5"])
    assert capsys.readouterr().out.startswith("hello there")


def test_causal_input_corruption_schedule_and_targets():
    import torch

    from burn_dragon_b200.config import CausalInputCorruptionConfig
    from burn_dragon_b200.train.corruption import corrupt_inputs

    c = CausalInputCorruptionConfig(enabled=True, probability=0.5, warmup_steps=2, ramp_steps=4)
    assert [c.probability_at(s) for s in (0, 1, 2, 3, 5, 9)] == [0.0, 0.0, 0.125, 0.25, 0.5, 0.5]
    x = torch.arange(4000).reshape(40, 100) % 200 + 10
    assert torch.equal(corrupt_inputs(x, c, 0, 256), x)
    y = corrupt_inputs(x, c, 9, 256, seed=1)
    frac = float((y != x).float().mean())
    assert 0.4 < frac < 0.52  # a random replacement can equal the original token
    c.replacement_token_id = 0
    z = corrupt_inputs(x, c, 9, 256, seed=1)
    assert set(z[z != x].tolist()) == {0} and torch.equal(z, corrupt_inputs(x, c, 9, 256, seed=1))


def test_separate_validation_source(tmp_path, monkeypatch, capsys):
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    train = tmp_path / "train.bin"
    np.full(20_000, ord("a"), dtype=np.uint8).tofile(train)
    held = tmp_path / "held.jsonl"
    held.write_text("\n".join(json.dumps({"text": "zq" * 300}) for _ in range(20)))
    base = ["--config", CFG, "--set", 'dataset.type="file"', "--set", f'dataset.path="{train}"',
            "--set", "training.max_iters=30", "--set", "training.validation_interval_iters=30",
            "--set", "training.block_size=32", "--set", "optimizer.learning_rate=0.01"]
    losses = {}
    for name, extra in (("same", []), ("held", ["--set", f'dataset.validation={{type="jsonl", path="{held}", '
                                                         f'cache_dir="{tmp_path / "vc"}"}}'])):
        main(base + extra + ["--run-name", name])
        res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
        ev = [json.loads(x) for x in open(os.path.join(res["run_dir"], "events", "metrics.jsonl"))]
        losses[name] = [e["valid_loss"] for e in ev if "valid_loss" in e][-1]
    # a model that learned "aaaa" scores its own split far better than unseen "zqzq" text
    assert losses["held"] > losses["same"] + 1.0
