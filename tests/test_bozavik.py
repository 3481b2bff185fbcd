"""Bozavik on the CPU: configuration, model as data, and the engine's step function, cache and trace replay with
the kernels' plain twins against the plain implementation."""

import io
import json

import numpy as np
import pytest
import torch

import bozavik_cases as cases
import helpers
import plain_bozavik
from torch_kernels import TorchKernels
from tt_transformers_b200.config import EngineConfig
from tt_transformers_b200.config.base import ConfigError
from tt_transformers_b200.engine.step import build_engine
from tt_transformers_b200.engine.trace import run_trace
from tt_transformers_b200.parts import DecoderModel, LatentPages
from tt_transformers_b200.registry import architecture_of, get_architecture


def test_configuration_reads_every_size_per_layer():
    arch = get_architecture(architecture_of(cases.ALIGNED))
    cfg = arch.load_config(cases.ALIGNED)
    assert [l.type for l in cfg.layers] == ["latent_attention_2", "latent_attention", "latent_attention", "latent_attention_2"]
    assert cfg.layers[3].mixer.rot_dim == 32 and cfg.layers[3].mixer.rot_dims == 16 and cfg.layers[2].mlp is None
    assert cfg.layers[1].mlp.shared_inter is None and cfg.layers[0].mlp.shared_limit == 0.8
    model = DecoderModel(arch.model_spec(cfg))
    assert model.cache_requests() == [LatentPages(64, 16), LatentPages(48, 0), LatentPages(32, 0), LatentPages(80, 32)]
    names = {s.name: s.shape for s in model.tensor_specs()}
    assert names["l0.mix.dkv"] == (64 + 16, 128) and names["l0.mix.g"] == (4, 128) and names["l1.mix.g"] == (3 * 32, 128)
    assert "l1.mix.sink" in names and "l0.mix.sink" not in names and "l2.mlp.router" not in names
    assert names["l3.mlp.shared.sg"] == (1, 128) and names["final.norm.b"] == (128,)


@pytest.mark.parametrize("breaker,match", [
    (lambda c: c["layers"][0].update(type="ring_attention"), "not known"),
    (lambda c: c["layers"][0]["mixer"].pop("kv_rank"), "kv_rank"),
    (lambda c: c["layers"][0]["mixer"]["rot"].update(dims=7), "rot.dims"),
    (lambda c: c["layers"][1]["mlp"]["router"].update(top=9), "top"),
    (lambda c: c.pop("norm"), "norm"),
])
def test_configuration_errors_name_the_key(breaker, match):
    cfg = json.loads(json.dumps(cases.ALIGNED))
    breaker(cfg)
    with pytest.raises(ConfigError, match=match):
        get_architecture("Bozavik").load_config(cfg)


@pytest.mark.parametrize("name", ["ALIGNED", "ODD"])
def test_engine_with_plain_twins_matches_the_plain_implementation(tmp_path, name):
    folder = cases.write_folder(str(tmp_path / name), getattr(cases, name), seed=3)
    cfg, w = cases.read_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(cfg["vocab"], n, 70 + i) for i, n in enumerate((37, 1, 19, 8, 26))}
    ref = {rid: plain_bozavik.forward(cfg, w, toks) for rid, toks in requests.items()}
    for make_steps in (helpers.steps_whole, helpers.steps_decode_tail, helpers.steps_portions, helpers.steps_mixed):
        steps = make_steps(requests)
        pages = -(-helpers.max_live_tokens(requests, steps, rounding=4) // 4)
        engine = build_engine(folder, EngineConfig(dtype="float32", page_size=4, num_pages=pages, max_batch_size=4,
                                                   max_seq_len=64, device="cpu"), kernels=TorchKernels())
        for g in engine.cache.groups:
            g.storage["rows"].fill_(float("nan"))           # a read of a row that was never written would show
        got = helpers.run_steps(engine, steps)
        engine.cache.audit()
        assert engine.cache.free_pages() == pages
        for rid in ref:
            assert helpers.relative_error(got[rid], ref[rid]) < 2e-5, (make_steps.__name__, rid)


def test_trace_replay_of_a_bozavik_folder(tmp_path):
    folder = cases.write_folder(str(tmp_path / "m"), cases.ODD, seed=5)
    cfg, w = cases.read_folder(folder)
    toks = helpers.random_tokens(cfg["vocab"], 15, 9)
    ref = plain_bozavik.forward(cfg, w, toks)
    lines = [{"step": 0, "entries": [{"id": "a", "tokens": toks[:9], "want": [0, 8]}], "end": []},
             {"step": 1, "entries": [{"id": "a", "tokens": toks[9:11], "want": []}], "end": []},
             {"step": 2, "entries": [{"id": "a", "tokens": toks[11:], "want": [3]}], "end": ["a"]}]
    log = io.StringIO()
    run_trace(folder, "float32", str(tmp_path / "out"), 64, [json.dumps(l) for l in lines], log=log, device="cpu",
              kernels=TorchKernels(), page_size=16)
    assert log.getvalue().split() == ["done", "0", "done", "1", "done", "2"]
    s0 = np.fromfile(tmp_path / "out" / "0.f32", dtype="<f4").reshape(2, cfg["vocab"])
    s2 = np.fromfile(tmp_path / "out" / "2.f32", dtype="<f4").reshape(1, cfg["vocab"])
    assert np.allclose(s0, ref[[0, 8]].numpy(), atol=2e-5) and np.allclose(s2, ref[[14]].numpy(), atol=2e-5)
    assert not (tmp_path / "out" / "1.f32").exists()


def test_the_plain_mechanisms_by_hand():
    """The oracle's own functions against loops written out element by element."""
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 10, generator=g)
    w, b = torch.randn(10, generator=g), torch.randn(10, generator=g)
    ln = plain_bozavik.layer_norm(x, w, b, 1e-3)
    for r in range(3):
        mean = sum(float(v) for v in x[r]) / 10
        var = sum((float(v) - mean) ** 2 for v in x[r]) / 10
        for c in range(10):
            assert abs(float(ln[r, c]) - ((float(x[r, c]) - mean) / (var + 1e-3) ** 0.5 * float(w[c]) + float(b[c]))) < 1e-5
    # rotation: dimension i pairs with i + dims/2; elements past `dims` pass unchanged
    v = torch.randn(2, 6, generator=g)
    out = plain_bozavik.rotate_halves(v, torch.tensor([0, 5]), 100.0, 4)
    assert torch.equal(out[0], v[0]) and torch.equal(out[:, 4:], v[:, 4:])
    a = 5 * 100.0 ** (-2 / 4)
    assert abs(float(out[1, 1]) - (float(v[1, 1]) * np.cos(a) - float(v[1, 3]) * np.sin(a))) < 1e-5
    assert abs(float(out[1, 3]) - (float(v[1, 3]) * np.cos(a) + float(v[1, 1]) * np.sin(a))) < 1e-5
    # a sink takes weight from the keys and gives it to nothing
    row = plain_bozavik.softmax_row_with_sink(torch.tensor([0.0, 0.0]), 0.0)
    assert torch.allclose(row, torch.tensor([1 / 3, 1 / 3]))
    # the expert: gate capped from above only, up clamped on both sides, (u + 1)
    y = plain_bozavik.clamped_expert(torch.tensor([[1.0]]), torch.tensor([[5.0], [-5.0]]), torch.tensor([[-9.0], [9.0]]),
                                     torch.eye(2), 2.0)
    s = 1 / (1 + np.exp(-1.702 * 2.0))
    s5 = 1 / (1 + np.exp(1.702 * 5.0))
    assert torch.allclose(y, torch.tensor([[2.0 * s * (-2.0 + 1.0), -5.0 * s5 * (2.0 + 1.0)]], dtype=torch.float32), atol=1e-5)


def test_greedy_generation_through_the_scheduler_under_page_pressure(tmp_path):
    from tt_transformers_b200.engine.llm import from_pretrained

    folder = cases.write_folder(str(tmp_path / "g"), cases.ODD, seed=7)
    cfg, w = cases.read_folder(folder)
    prompts = [helpers.random_tokens(cfg["vocab"], n, 80 + n) for n in (4, 13, 21)]

    def plain_greedy(prompt, new):
        toks = list(prompt)
        for _ in range(new):
            toks.append(int(plain_bozavik.forward(cfg, w, toks)[-1].argmax()))
        return toks[len(prompt):]

    expect = [plain_greedy(p, 6) for p in prompts]
    # 7 pages of 8 tokens for requests that end at 10, 19 and 27 tokens: they cannot all stay, one gives way and is recomputed
    llm = from_pretrained(folder, dtype="float32", page_size=8, num_pages=7, max_batch_size=3, max_seq_len=64,
                          max_step_tokens=16, max_chunk_tokens=8, device="cpu", kernels=TorchKernels())
    assert llm.generate(prompts, max_new_tokens=6) == expect
    llm.engine.cache.audit()
    assert llm.engine.cache.free_pages() == 7
