"""Burnpack bootstrap: resolve weights from the cache or fetch them (parts first, then the
monolithic file) from a base URL, over file:// and a loopback HTTP server."""
import functools
import http.server
import os
import threading

import pytest
import torch

from burn_dragon_b200.train import burnpack as BP


def _remote(tmp_path, parts: bool):
    src = tmp_path / "remote"
    src.mkdir()
    t = {"a": torch.arange(1000, dtype=torch.float32), "b": torch.ones(300, 7)}
    BP.save_burnpack(str(src / "model.bpk"), t, {"k": "v"})
    if parts:
        BP.write_parts(str(src / "model.bpk"), max_part_mib=1)
    return src, t


def test_candidate_urls_follow_precision_preference():
    assert BP.candidate_urls("https://h/m/model") == ["https://h/m/model.bpk", "https://h/m/model_f16.bpk"]
    assert BP.candidate_urls("https://h/m/model.bpk", prefer_f16=True)[0] == "https://h/m/model_f16.bpk"


def test_cache_root_env_override(monkeypatch, tmp_path):
    monkeypatch.setenv("BURN_DRAGON_CACHE_DIR", str(tmp_path / "c"))
    assert BP.default_cache_root() == str(tmp_path / "c")


@pytest.mark.parametrize("parts", [True, False])
def test_bootstrap_over_file_urls(tmp_path, parts):
    src, t = _remote(tmp_path, parts)
    os.remove(src / "model.bpk") if parts else None  # parts alone must suffice
    cache = tmp_path / "cache"
    msgs = []
    p = BP.resolve_or_bootstrap("m/model", "file://" + str(src / "model"), cache_root=str(cache),
                                progress=msgs.append)
    assert p == str(cache / "m" / "model.bpk")
    got, meta = BP.load_resolved(p)
    assert torch.equal(got["a"], t["a"]) and torch.equal(got["b"], t["b"]) and meta["k"] == "v"
    assert BP.manifest_complete(BP.parts_manifest_path(p)) == parts
    # second resolve: served from the cache, no download
    msgs.clear()
    assert BP.resolve_or_bootstrap("m/model", "file:///nonexistent/model", cache_root=str(cache),
                                   progress=msgs.append) == p
    assert msgs and msgs[0].startswith("using cached")


def test_bootstrap_rejects_corrupt_part_then_falls_back(tmp_path):
    src, t = _remote(tmp_path, parts=True)
    man = BP.parts_manifest_path(str(src / "model.bpk"))
    import json

    m = json.load(open(man))
    first = src / m["parts"][0]["path"]
    first.write_bytes(b"\0" * first.stat().st_size)  # same size, wrong checksum
    cache = tmp_path / "cache"
    p = BP.resolve_or_bootstrap("model", "file://" + str(src / "model"), cache_root=str(cache))
    got, _ = BP.load_resolved(p)  # the monolithic file
    assert torch.equal(got["a"], t["a"])
    assert not BP.manifest_complete(BP.parts_manifest_path(p))


def test_bootstrap_over_loopback_http(tmp_path):
    src, t = _remote(tmp_path, parts=True)
    handler = functools.partial(http.server.SimpleHTTPRequestHandler, directory=str(src))
    handler.log_message = lambda *a, **k: None
    srv = http.server.ThreadingHTTPServer(("127.0.0.1", 0), handler)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    try:
        url = f"http://127.0.0.1:{srv.server_address[1]}/model"
        p = BP.resolve_or_bootstrap("model", url, cache_root=str(tmp_path / "cache"))
        got, _ = BP.load_resolved(p)
        assert torch.equal(got["b"], t["b"])
        with pytest.raises(FileNotFoundError):
            BP.resolve_or_bootstrap("other", f"http://127.0.0.1:{srv.server_address[1]}/missing",
                                    cache_root=str(tmp_path / "cache"))
    finally:
        srv.shutdown()


def test_generate_cli_loads_bootstrapped_weights(tmp_path, monkeypatch, capsys):
    """Train a tiny run, export its weights as parts, and generate from a fresh run dir
    whose weights come through --weights-url (file://)."""
    import json

    from burn_dragon_b200.cli.generate import main as gen
    from burn_dragon_b200.cli.train import main as train_main
    from burn_dragon_b200.models.bdh import BDH
    from burn_dragon_b200.train.checkpoint import RunDir, export_burnpack
    from burn_dragon_b200.config import training_config_from_dict

    cfgs = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")
    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path / "runs"))
    train_main(["--config", cfgs, "--set", "training.max_iters=2", "--set", "training.checkpoint_interval_iters=2",
                "--run-name", "g"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    run = RunDir(res["run_dir"])
    cfg = training_config_from_dict(run.read_json("training_config.json"))
    model = BDH(cfg.model, device="cpu")
    run.load(None, model)
    export_burnpack(model, str(tmp_path / "pub" / "tiny"), part_mib=1)
    gen(["--run", res["run_dir"], "--prompt", "ab", "--max-tokens", "4", "--output-format", "token_ids",
         "--weights-url", "file://" + str(tmp_path / "pub" / "tiny"), "--weights-cache", str(tmp_path / "wc")])
    a = capsys.readouterr().out.strip().splitlines()[-1]
    gen(["--run", res["run_dir"], "--prompt", "ab", "--max-tokens", "4", "--output-format", "token_ids"])
    b = capsys.readouterr().out.strip().splitlines()[-1]
    assert json.loads(a) == json.loads(b)  # same weights, same greedy / seeded tokens
    assert os.path.exists(tmp_path / "wc" / "tiny.bpk.parts.json")
