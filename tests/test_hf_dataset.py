"""Hugging Face dataset sources read from the local hub cache (no network): snapshot
resolution, file discovery, record rendering, pre-tokenised ids and the training loop."""
import json
import os

import numpy as np
import pytest

from burn_dragon_b200.train import datasets as DS


def _hub(tmp_path, repo_id, files: dict, rev="abc123", ref="main"):
    root = tmp_path / "cache" / "huggingface" / ("datasets--" + repo_id.replace("/", "--"))
    snap = root / "snapshots" / rev
    for rel, content in files.items():
        p = snap / rel
        p.parent.mkdir(parents=True, exist_ok=True)
        if isinstance(content, bytes):
            p.write_bytes(content)
        else:
            p.write_text(content)
    (root / "refs").mkdir(parents=True, exist_ok=True)
    (root / "refs" / ref).write_text(rev)
    return str(tmp_path / "cache"), str(snap)


def test_snapshot_resolution_and_discovery(tmp_path):
    cache, snap = _hub(tmp_path, "org/set", {"data/train-0.jsonl": "{}\n", "data/test-0.jsonl": "{}\n",
                                             "README.md": "x"})
    assert DS.hf_snapshot_root("org/set", None, cache) == snap
    assert DS.hf_snapshot_root("org/set", "abc123", cache) == snap  # a snapshot id as revision
    spec = DS.hf_defaults({"repo_id": "org/set", "auto_discover_train_files": True})
    assert DS.hf_files(spec, snap) == ["data/train-0.jsonl"]  # "train" paths preferred
    assert DS.hf_defaults({"repo_id": "a/b"})["train_files"] == ["train.jsonl"]
    with pytest.raises(FileNotFoundError):
        DS.hf_snapshot_root("org/missing", None, cache)


def test_record_rendering():
    spec = DS.hf_defaults({"repo_id": "a/b", "text_fields": ["q", "a"], "field_separator": " | "})
    assert DS.render_record(spec, {"q": "hi", "a": "there"}) == "hi | there"
    assert DS.render_record(spec, {"q": "hi"}) is None
    spec = DS.hf_defaults({"repo_id": "a/b", "template": "{prompt}\n\n{answer}"})
    assert DS.render_record(spec, {"prompt": "p", "answer": "a"}) == "p\n\na"
    with pytest.raises(ValueError):
        DS.render_record(DS.hf_defaults({"repo_id": "a/b", "template": "{x"}), {"x": 1})


def test_prepare_jsonl_and_parquet_ids(tmp_path):
    recs = "\n".join(json.dumps({"text": t}) for t in ["alpha", "beta", "gamma"]) + "\n"
    cache, _ = _hub(tmp_path, "org/txt", {"train.jsonl": recs, "valid.jsonl": recs})
    out = DS.prepare_hf_dataset({"repo_id": "org/txt", "max_records": 2, "field_separator": "\n"}, cache)
    assert open(out, "rb").read() == b"alpha\nbeta"
    assert DS.token_bytes(out) == 1
    assert DS.prepare_hf_dataset({"repo_id": "org/txt", "max_records": 2, "field_separator": "\n"}, cache) == out
    val = DS.prepare_hf_dataset({"repo_id": "org/txt", "validation_files": ["valid.jsonl"]}, cache, split="validation")
    assert open(val, "rb").read() == b"alpha\n\nbeta\n\ngamma"

    import pyarrow as pa
    import pyarrow.parquet as pq

    cache2 = tmp_path / "c2"
    root = cache2 / "huggingface" / "datasets--nvidia--Nemotron-CC--data--climb_mix" / "snapshots" / "r1"
    (root / "default").mkdir(parents=True)
    pq.write_table(pa.table({"input_ids": [[1, 2, 3], [400, 65535]]}), str(root / "default" / "part-0.parquet"))
    out = DS.prepare_hf_dataset({"type": "nemotron_climb_mix"}, str(cache2))
    assert DS.token_bytes(out) == 2
    assert np.fromfile(out, dtype="<u2").tolist() == [1, 2, 3, 400, 65535]


def test_training_loop_reads_a_huggingface_source(tmp_path, monkeypatch, capsys):
    from burn_dragon_b200.cli.train import main

    text = "\n".join(json.dumps({"text": "the quick brown fox " * 20}) for _ in range(20)) + "\n"
    cache, _ = _hub(tmp_path, "org/fox", {"train.jsonl": text})
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path / "runs"))
    cfgp = tmp_path / "hf.toml"
    cfgp.write_text(f"""
extends = "{os.path.join(os.path.dirname(__file__), '..', 'burn_dragon_b200', 'configs', 'tiny_cpu.toml').replace(os.sep, '/')}"
[dataset]
type = "huggingface"
cache_dir = "{cache.replace(os.sep, '/')}"
huggingface = {{ repo_id = "org/fox" }}
[training]
max_iters = 3
""")
    main(["--config", str(cfgp), "--run-name", "hf"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    losses = [json.loads(line)["loss"] for line in open(os.path.join(res["run_dir"], "events", "metrics.jsonl"))
              if "loss" in line]
    assert losses and all(np.isfinite(v) for v in losses)
    assert any(f.startswith("hf-") and f.endswith(".bin") for f in os.listdir(cache))
