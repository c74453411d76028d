"""Checkpoint round trips (CPU): tensor files, parts, precision, run dir, resume."""
import os

import torch

from burn_dragon_b200.config import DragonConfig, TrainingConfig
from burn_dragon_b200.models.bdh import BDH
from burn_dragon_b200.train import checkpoint as C
from burn_dragon_b200.train.optim import FusedAdamW


def _cfg():
    return DragonConfig(n_layer=2, n_embd=32, n_head=2, mlp_internal_dim_multiplier=4, dropout=0.0,
                        rotary_embedding="rope")


def test_tensor_file_round_trip(tmp_path):
    t = {"a": torch.randn(3, 4), "b": torch.arange(5), "c": torch.randn(2).bfloat16(), "e": torch.empty(0)}
    p = str(tmp_path / "x.bin")
    C.save_tensors(p, t, {"step": 7, "name": "x"})
    back, meta = C.load_tensors(p)
    assert meta == {"step": 7, "name": "x"}
    for k in t:
        assert back[k].dtype == t[k].dtype and torch.equal(back[k], t[k])


def test_parts_and_precision(tmp_path):
    t = {f"w{i}": torch.randn(64, 64) for i in range(5)}
    p = str(tmp_path / "model.bin")
    man = C.save_parts(p, t, max_part_bytes=2 * 64 * 64 * 4)
    assert len(man["parts"]) == 3
    back = C.load_parts(p)
    assert all(torch.equal(back[k], t[k]) for k in t)
    h = C.convert_precision(t, torch.float16)
    assert all(v.dtype == torch.float16 for v in h.values())


def test_run_dir_resume_preserves_logits_and_optimizer(tmp_path):
    cfg = _cfg()
    model = BDH(cfg, seed=3)
    opt = FusedAdamW(model.store, lr=1e-2)
    x = torch.randint(0, 256, (2, 8))
    y = torch.randint(0, 256, (2, 8))
    for _ in range(2):
        loss = model.loss(x, y)
        grads = torch.autograd.grad(loss, list(model.parameters()), allow_unused=True)
        for p, g in zip(model.parameters(), grads):
            if g is not None:
                p.grad.copy_(g)
        opt.step()
    run = C.RunDir(C.resolve_run_dir("cpu", "t", root=str(tmp_path)))
    tc = TrainingConfig(model=cfg)
    run.write_run_config(tc)
    rho = [torch.randn(2, 2, 32, 32) for _ in range(2)]
    run.save(2, model, opt, {"step": 2}, {"position": 8, "rhos": rho})
    assert os.path.exists(os.path.join(run.path, "config.json"))
    model2 = BDH(cfg, seed=99)
    opt2 = FusedAdamW(model2.store, lr=1e-2)
    info = run.load(None, model2, opt2)
    assert info["step"] == 2 and info["runtime"]["position"] == 8
    assert torch.equal(info["runtime"]["rhos"][1], rho[1])
    assert torch.allclose(model(x), model2(x))
    assert opt2.t == opt.t and torch.equal(opt2.m, opt.m)


def test_retention_keeps_last_two_and_best(tmp_path):
    model = BDH(_cfg(), seed=1)
    run = C.RunDir(str(tmp_path / "r"))
    for s in (1, 2, 3, 4):
        run.save(s, model, best_step=1)
    assert run.steps() == [1, 3, 4]
    assert run.latest() == 4


def test_async_write_snapshots_before_training_continues(tmp_path):
    cfg = DragonConfig(n_layer=1, n_embd=32, n_head=2, mlp_internal_dim_multiplier=2, dropout=0.0, vocab_size=64)
    model = BDH(cfg, seed=5)
    opt = FusedAdamW(model.store, lr=1e-2)
    run = C.RunDir(os.path.join(str(tmp_path), "a"), async_write=True)
    want = model.store.data.clone()
    run.save(1, model, opt, {"step": 1})
    model.store.data.add_(1.0)  # training goes on while the files are written
    run.save(2, model, opt, {"step": 2})
    run.wait()
    assert run.latest() == 2 and run.steps() == [1, 2]
    m2 = BDH(cfg, seed=6)

    def params(buf):  # the parameter views (the flat store also holds alignment padding)
        return m2.store.views(buf)

    run.load(1, m2)
    for n, v in params(m2.store.data).items():
        torch.testing.assert_close(v, params(want)[n])
    run.load(2, m2)
    for n, v in params(m2.store.data).items():
        torch.testing.assert_close(v, params(want)[n] + 1.0)


def test_training_with_async_checkpoints(tmp_path, monkeypatch, capsys):
    import json

    from burn_dragon_b200.cli.train import main

    monkeypatch.setenv("BURN_DRAGON_RUN_ROOT", str(tmp_path))
    cfg = os.path.join(os.path.dirname(__file__), "..", "burn_dragon_b200", "configs", "tiny_cpu.toml")
    main(["--config", cfg, "--set", "training.max_iters=4", "--set", "training.checkpoint_interval_iters=2",
          "--set", "parallel.checkpoint={async_write=true}", "--run-name", "aw"])
    res = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert os.path.exists(os.path.join(res["run_dir"], "checkpoint", "model-4.bpk"))
    assert open(os.path.join(res["run_dir"], "latest")).read().strip() == "4"


def test_runtime_state_with_auxiliary_memories_round_trips(tmp_path):
    from burn_dragon_b200.models.dragon_runtime import LayerState, RuntimeState

    st = RuntimeState([LayerState(rho=torch.randn(1, 2, 4, 8), y_state=torch.randn(1, 2, 4)),
                       LayerState(summary_hidden=torch.randn(1, 1, 8), mamba={"ssm": torch.randn(1, 2, 3)})], 17)
    cfg = DragonConfig(n_layer=2, n_embd=8, n_head=2, mlp_internal_dim_multiplier=2, dropout=0.0, vocab_size=16)
    run = C.RunDir(os.path.join(str(tmp_path), "r"))
    run.save(1, BDH(cfg, seed=1), None, {"step": 1},
             {"position": st.position, "state_tensors": st.to_tensors()})
    info = run.load(1, BDH(cfg, seed=2))
    back = RuntimeState.from_tensors(2, info["runtime"]["state_tensors"], int(info["runtime"]["position"]))
    assert back.position == 17 and back.layers[0].clocked_hidden is None
    torch.testing.assert_close(back.layers[0].rho, st.layers[0].rho)
    torch.testing.assert_close(back.layers[0].y_state, st.layers[0].y_state)
    torch.testing.assert_close(back.layers[1].summary_hidden, st.layers[1].summary_hidden)
    torch.testing.assert_close(back.layers[1].mamba["ssm"], st.layers[1].mamba["ssm"])
    assert info["runtime"]["rhos"] is None


def _burnpack_vector(tmp_path):
    """A burnpack file assembled byte by byte from the format's definition (header of
    magic 0x4255524E, u16 version, u32 CBOR size; CBOR {"tensors", "metadata"}; data at
    the next 256-byte boundary, each payload 256-aligned), independent of the writer."""
    import struct

    a = torch.arange(6, dtype=torch.float32).reshape(2, 3)
    b = torch.tensor([1, -2], dtype=torch.int64)

    def text(s):
        raw = s.encode()
        assert len(raw) < 24
        return bytes([0x60 | len(raw)]) + raw

    def uint(n):
        return bytes([n]) if n < 24 else (bytes([0x18, n]) if n < 256 else bytes([0x19]) + struct.pack(">H", n))

    def arr(items):
        return bytes([0x80 | len(items)]) + b"".join(items)

    def desc(dtype, shape, lo, hi):
        return (bytes([0xA3]) + text("dtype") + text(dtype) + text("shape") + arr([uint(s) for s in shape])
                + text("data_offsets") + arr([uint(lo), uint(hi)]))

    cbor = (bytes([0xA2]) + text("tensors") + bytes([0xA2]) + text("a") + desc("F32", [2, 3], 0, 24)
            + text("b") + desc("I64", [2], 256, 272) + text("metadata") + bytes([0xA1]) + text("k") + text("v"))
    head = struct.pack("<IHI", 0x4255524E, 1, len(cbor))
    start = -(-(len(head) + len(cbor)) // 256) * 256
    data = bytearray(start + 272)
    data[:len(head)] = head
    data[len(head):len(head) + len(cbor)] = cbor
    data[start:start + 24] = a.numpy().tobytes()
    data[start + 256:start + 272] = b.numpy().tobytes()
    p = tmp_path / "vec.bpk"
    p.write_bytes(bytes(data))
    return str(p), a, b


def test_burnpack_reader_parses_a_spec_test_vector(tmp_path):
    from burn_dragon_b200.train import burnpack as BP

    p, a, b = _burnpack_vector(tmp_path)
    t, meta = BP.load_burnpack(p)
    assert meta == {"k": "v"}
    assert torch.equal(t["a"], a) and torch.equal(t["b"], b)
    # the writer lays the same tensors out identically (same offsets, same payload bytes)
    q = str(tmp_path / "out.bpk")
    BP.save_burnpack(q, {"a": a, "b": b}, {"k": "v"})
    _, _, md = BP.read_header(q)
    assert md["tensors"]["a"]["data_offsets"] == [0, 24] and md["tensors"]["b"]["data_offsets"] == [256, 272]
    assert open(q, "rb").read() == open(p, "rb").read()


def test_burnpack_round_trip_parts_and_f16(tmp_path):
    from burn_dragon_b200.train import burnpack as BP

    t = {f"w{i}": torch.randn(300, 512) for i in range(5)}  # 600 KiB each
    t["ids"] = torch.arange(10)
    t["h"] = torch.randn(7).bfloat16()
    p = str(tmp_path / "model.bpk")
    BP.save_burnpack(p, t, {"step": "3"})
    back, meta = BP.load_burnpack(p)
    assert meta == {"step": "3"} and all(torch.equal(back[k], t[k]) for k in t)
    man = BP.write_parts(p, max_part_mib=1)
    assert len(man["parts"]) == 5 and sum(e["tensors"] for e in man["parts"]) == len(t)
    assert all(len(e["sha256"]) == 64 and e["path"].endswith(".bpk") for e in man["parts"])
    back2, _ = BP.load_parts(BP.parts_manifest_path(p))
    assert all(torch.equal(back2[k], t[k]) for k in t)
    # a corrupted part is refused
    part = tmp_path / man["parts"][0]["path"]
    raw = bytearray(part.read_bytes())
    raw[-1] ^= 0xFF
    part.write_bytes(bytes(raw))
    import pytest

    with pytest.raises(ValueError):
        BP.load_parts(BP.parts_manifest_path(p))
    # f16 variant: floats converted, integers kept, precision recorded
    h = BP.convert_precision(p, BP.precision_path(p, True), "f16")
    assert h.endswith("model_f16.bpk")
    th, mh = BP.load_burnpack(h)
    assert mh["precision"] == "f16" and th["w0"].dtype == torch.float16 and th["ids"].dtype == torch.int64


def test_model_burnpack_export_and_load(tmp_path):
    cfg = _cfg()
    m1, m2 = BDH(cfg, seed=1), BDH(cfg, seed=2)
    out = C.export_burnpack(m1, str(tmp_path / "deploy"), part_mib=1)
    assert out.endswith("deploy.bpk")
    C.load_model_burnpack(m2, out)
    assert torch.equal(m1.store.data, m2.store.data)
    f16 = C.export_burnpack(m1, str(tmp_path / "deploy"), f16=True)
    m3 = BDH(cfg, seed=3)
    assert C.load_model_burnpack(m3, str(tmp_path / "deploy.bpk"), prefer_f16=True) == f16
    assert torch.allclose(m3.store.data, m1.store.data, atol=1e-3)


def test_sharded_v2_records_reassemble_for_any_world(tmp_path):
    """Two ranks each write their own slices of master / moments (sharded_v2); a load
    assembles the full store and moments, and refuses an incomplete shard set."""
    import pytest

    cfg = _cfg()
    model = BDH(cfg, seed=3)
    opt = FusedAdamW(model.store, lr=1e-2)
    n = model.store.numel
    opt.m.copy_(torch.randn(n))
    opt.v.copy_(torch.rand(n))
    opt.t = 5
    run = C.RunDir(str(tmp_path / "r"))
    # rank r owns two interleaved slices (the NVLink step's per-bucket layout)
    half, q = n // 2, n // 4
    owned = {0: [(0, q), (half, half + q)], 1: [(q, half), (half + q, n)]}
    for r, sl in owned.items():
        cat = lambda t: torch.cat([t[a:b] for a, b in sl])  # noqa: E731
        run.save_shard(4, r, 2, sl, model.store.data, cat(opt.m), cat(opt.v), n, opt.t)
    run.save(4, model, opt, {"step": 4}, sharded=True)
    assert run.latest() == 4 and run.steps() == [4]
    m2 = BDH(cfg, seed=99)
    o2 = FusedAdamW(m2.store, lr=1e-2)
    run.load(None, m2, o2)
    assert torch.equal(m2.store.data, model.store.data)
    assert torch.equal(o2.m, opt.m) and torch.equal(o2.v, opt.v) and o2.t == 5
    os.remove(run.shard_files(4)[1])
    with pytest.raises(ValueError):
        run.load(4, m2, o2)
