"""Pedazen on the CPU: configuration, model as data, and the engine's step function, cache manager, scheduler and
trace replay with the kernels' plain twins against the plain implementation."""

import io
import json
import math

import numpy as np
import pytest
import torch

import helpers
import pedazen_cases as cases
import plain_pedazen
from torch_kernels import TorchKernels
from tt_transformers_b200.config import EngineConfig
from tt_transformers_b200.config.base import ConfigError
from tt_transformers_b200.engine.step import StepEntry, build_engine
from tt_transformers_b200.engine.trace import run_trace
from tt_transformers_b200.parts import DecoderModel, PagedKV, SlotState
from tt_transformers_b200.parts.base import RecurrentState
from tt_transformers_b200.registry import architecture_of, get_architecture


def _plain(cfg, w, toks):
    return plain_pedazen.forward(cfg, w, toks).float()


def _engine(folder, pages, page_size=4, slots=4, max_seq_len=128, **more):
    return build_engine(folder, EngineConfig(dtype="float32", page_size=page_size, num_pages=pages, max_batch_size=slots,
                                             max_seq_len=max_seq_len, device="cpu", **more), kernels=TorchKernels())


def _poison(engine):
    """What a page or a slot held before must never be read: NaN everywhere (admission zeroes a slot's state)."""
    for g in engine.cache.groups:
        for t in g.storage.values():
            t.fill_(float("nan"))


def test_configuration_and_model_as_data():
    arch = get_architecture(architecture_of(cases.ALIGNED))
    cfg = arch.load_config(cases.ALIGNED)
    assert [l.type for l in cfg.layers] == ["parallel", "lightning", "parallel", "lightning"]
    assert (cfg.loop_start, cfg.loop_stop, cfg.loop_times) == (1, 3, 3)
    assert cfg.layers[2].mixer.left.kv_heads == 1 and cfg.layers[2].mixer.left.softcap == 5.0 and cfg.layers[2].mlp is None
    assert cfg.layers[1].mlp.groups == 4 and cfg.layers[1].mlp.keep == 2 and cfg.layers[0].mlp.kind == "dense"
    spec = arch.model_spec(cfg)
    assert [c.layer for c in spec.order] == [0, 1, 2, 1, 2, 1, 2, 3]
    assert [at for at, _ in spec.stream_steps] == [1, 3, 5]
    assert [s.params["add_embedding"] for _, s in spec.stream_steps] == [False, True, True]
    model = DecoderModel(spec)
    requests = model.cache_requests()
    assert requests[0] == (PagedKV(2, 32, None, value_dim=16, chunk=24), RecurrentState(96, 3))
    assert requests[1] == requests[3] == requests[5] == SlotState((2, 48, 32), torch.float32)     # a state per pass
    assert requests[7] == SlotState((3, 16, 64), torch.float32)
    names = {s.name: s.shape for s in model.tensor_specs()}
    assert names["loop.step"] == (3, 128) and names["l0.mix.right.ra"] == (3, 32, 32) and names["l0.mix.left.sink"] == (4,)
    assert names["l2.mix.left.k"] == (16, 128) and names["l2.mix.left.v"] == (48, 128) and names["l2.mix.left.o"] == (128, 288)
    assert names["l1.mlp.e7.up"] == (48, 128) and "l2.mlp.router" not in names and "head" not in names
    assert names["l0.mix.left.out"] == (128,) and names["l0.mix.right.conv"] == (96, 3) and names["l3.mix.norm"] == (192,)
    # a model without a loop has neither passes nor their table
    plain_spec = arch.model_spec(arch.load_config(cases.PLAIN))
    assert plain_spec.stream_steps == () and "loop.step" not in {s.name for s in DecoderModel(plain_spec).tensor_specs()}
    # cut short, the model keeps the passes that still start
    assert [at for at, _ in spec.first_entries(4).stream_steps] == [1, 3]


@pytest.mark.parametrize("breaker,match", [
    (lambda c: c["layers"][0].update(type="ring"), "not known"),
    (lambda c: c["layers"][1]["mixer"].pop("decay"), "decay"),
    (lambda c: c["layers"][1]["mixer"].update(decay=[0.5]), "decays for"),
    (lambda c: c["layers"][0]["mixer"]["left"]["rot"].update(dims=7), "rot.dims"),
    (lambda c: c["layers"][0]["mixer"]["left"].update(kv_heads=3), "kv_heads"),
    (lambda c: c["layers"][0]["mixer"]["right"].update(blocks=5), "blocks"),
    (lambda c: c["layers"][1]["mlp"]["router"].update(top=9), "top"),
    (lambda c: c["layers"][1]["mlp"]["router"]["groups"].update(count=3), "groups.count"),
    (lambda c: c["layers"][3]["mlp"]["router"].update(top=4), "fewer than 'top'"),
    (lambda c: c["loop"].update(stop=9), "loop"),
    (lambda c: c.pop("norm"), "norm"),
])
def test_configuration_errors_name_the_key(breaker, match):
    cfg = json.loads(json.dumps(cases.ALIGNED))
    breaker(cfg)
    with pytest.raises(ConfigError, match=match):
        get_architecture("Pedazen").load_config(cfg)


@pytest.mark.parametrize("kind", ["lightning", "parallel", "dense", "moe"])
def test_each_mechanism_alone(tmp_path, kind):
    folder = cases.write_folder(str(tmp_path / kind), cases.single(kind), seed=11)
    cfg, w = cases.read_folder(folder)
    requests = {"a": helpers.random_tokens(cfg["vocab"], 33, 1), "b": helpers.random_tokens(cfg["vocab"], 12, 2)}
    ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
    for make_steps in (helpers.steps_whole, helpers.steps_portions, helpers.steps_decode_tail):
        engine = _engine(folder, pages=12)
        _poison(engine)
        got = helpers.run_steps(engine, make_steps(requests))
        for rid in ref:
            assert helpers.relative_error(got[rid], ref[rid]) < 2e-5, (make_steps.__name__, rid)


@pytest.mark.parametrize("name", ["ALIGNED", "ODD", "PLAIN"])
def test_engine_with_plain_twins_matches_the_plain_implementation(tmp_path, name):
    """Whole prompts, prompts with decoded tails, portions down to two tokens, and mixed batches of unequal requests
    on a pool that holds just what is live, with five requests on four slots: pages and slots are used again."""
    folder = cases.write_folder(str(tmp_path / name), getattr(cases, name), seed=3)
    cfg, w = cases.read_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(cfg["vocab"], n, 70 + i) for i, n in enumerate((37, 1, 19, 8, 26, 2))}
    ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
    for make_steps in (helpers.steps_whole, helpers.steps_decode_tail, helpers.steps_portions, helpers.steps_mixed):
        steps = make_steps(requests)
        pages = -(-helpers.max_live_tokens(requests, steps, rounding=4) // 4)
        engine = _engine(folder, pages=pages, max_seq_len=64)
        _poison(engine)
        got = helpers.run_steps(engine, steps)
        engine.cache.audit()
        assert engine.cache.free_pages() == pages and engine.cache.free_slots == 4
        for rid in ref:
            assert helpers.relative_error(got[rid], ref[rid]) < 2e-5, (make_steps.__name__, rid)


def test_pages_behind_the_current_chunk_are_given_back(tmp_path):
    """Chunks of 16 positions (layer 2) and of 24 (layer 0) on pages of 4: a request of 70 tokens never holds
    more pages per group than its current chunk needs, plus the token that may be taken back."""
    folder = cases.write_folder(str(tmp_path / "m"), cases.ALIGNED, seed=5)
    cfg, w = cases.read_folder(folder)
    toks = helpers.random_tokens(cfg["vocab"], 70, 4)
    ref = _plain(cfg, w, toks)
    engine = _engine(folder, pages=14, max_seq_len=128)         # 70 tokens would need 18 pages without giving back
    _poison(engine)
    rows, at = [], 0
    for n in [5, 2, 9, 1, 1, 17, 3, 1, 1, 1, 2, 20, 1, 1, 5]:
        rows.append(engine.step([StepEntry("a", toks[at:at + n], list(range(n)))]))
        at += n
        assert engine.cache.free_pages() >= 14 - 8             # a chunk of 24 positions on pages of 4, and the token before
    assert at == 70
    assert helpers.relative_error(torch.cat(rows), ref) < 2e-5
    engine.finish("a")
    engine.cache.audit()
    assert engine.cache.free_pages() == 14


def _scores_setup(kernels, device, chunk, softcap, page, pos0, new, heads=2, kv_heads=1, dim=8, vdim=4, window=None):
    """One request with pos0 cached tokens and `new` new ones whose keys are all zero but chosen ones: returns what a
    test needs to write keys through the kernel table and attend."""
    from types import SimpleNamespace

    ctx = pos0 + new
    n_pages = -(-ctx // page)
    order = list(range(n_pages, 0, -1))                         # pages in descending order: the table is used
    keys = torch.full((n_pages + 1, kv_heads, page, dim), float("nan"), device=device)
    values = torch.full((n_pages + 1, kv_heads, page, vdim), float("nan"), device=device)
    table = torch.tensor([order], dtype=torch.int32, device=device)
    view = PagedKV(kv_heads, dim, window, value_dim=vdim, chunk=chunk).view({"keys": keys, "values": values}, block_table=table,
                                                                            page_size=page)

    def batch(p0, n):
        return SimpleNamespace(positions=torch.arange(p0, p0 + n, dtype=torch.int32, device=device),
                               seg_of_token=torch.zeros(n, dtype=torch.int32, device=device), seg_lens=[n], seg_pos0_list=[p0],
                               cu_seqlens=torch.tensor([0, n], dtype=torch.int32, device=device), num_segments=1)
    return view, batch


def check_one_key_carries_the_weight(kernels, device, dtype=torch.float32):
    """A query whose score with one key stands out returns that key's value, if the key lies in the query's chunk
    (its first position, a page's edge, the query's own position), and nothing of it if it lies just outside;
    for a decoded token and for the last token of a portion."""
    heads, kv_heads, dim, vdim, page, chunk = 2, 1, 8, 4, 4, 12
    for pos0, new in ((40, 1), (38, 3), (36, 1), (35, 2), (0, 30)):
        last = pos0 + new - 1
        start = last // chunk * chunk
        for far in sorted({start, start - 1, last, max(start, last - 1), (start // page + 1) * page, (start // page + 1) * page - 1}):
            if far < 0 or far > last:
                continue
            view, batch = _scores_setup(kernels, device, chunk, 30.0, page, pos0, new, heads, kv_heads, dim, vdim)
            view.keys, view.values = view.keys.to(dtype), view.values.to(dtype)
            ctx = pos0 + new
            g = torch.Generator().manual_seed(far)
            k_all = torch.zeros(ctx, kv_heads * dim)
            k_all[far, 0] = 6.0
            v_all = torch.randn(ctx, kv_heads * vdim, generator=g)
            q = torch.zeros(ctx, heads * dim)
            q[:, 0] = 6.0
            q[:, dim] = 6.0
            qkv = torch.cat([q, k_all, v_all], 1).to(device, dtype)
            if pos0:
                head = qkv[:pos0].clone()
                kernels.qk_norm_rope_write(head, batch(0, pos0), None, None, 1e-6, None, 0, heads, kv_heads, dim, vdim, view)
            tail = qkv[pos0:].clone()
            kernels.qk_norm_rope_write(tail, batch(pos0, new), None, None, 1e-6, None, 0, heads, kv_heads, dim, vdim, view)
            out = kernels.sink_attention(tail, batch(pos0, new), heads, kv_heads, dim, vdim, 1.0, 30.0, None, view)
            got = out[-1].float().cpu().view(heads, vdim)
            assert not torch.isnan(got).any()
            if far >= start:                    # capped at 30 against zeros: the weight of all others is below 1e-11
                assert torch.allclose(got, v_all[far].to(dtype).float().view(1, vdim).expand(heads, vdim), atol=2e-2 if dtype != torch.float32 else 1e-5), (pos0, new, far)
            else:                               # outside: the mean of the chunk's values, the far one not among them
                mean = v_all[start:last + 1].to(dtype).float().mean(0)
                assert torch.allclose(got, mean.view(1, vdim).expand(heads, vdim), atol=2e-2 if dtype != torch.float32 else 1e-5), (pos0, new, far)


def test_one_key_carries_the_weight_inside_its_chunk_only():
    check_one_key_carries_the_weight(TorchKernels(), "cpu")


def test_the_plain_mechanisms_by_hand():
    """The oracle's own functions against numbers worked out by hand."""
    # RMS norm: eps inside the root
    x = torch.tensor([[3.0, 4.0]], dtype=torch.float64)
    assert torch.allclose(plain_pedazen.rms(x, 0.5), x / math.sqrt(12.5 + 0.5))
    # rotation: element i pairs with i + dims/2, elements past dims pass unchanged, position 0 changes nothing
    v = torch.arange(1.0, 13.0, dtype=torch.float64).view(2, 1, 6)
    out = plain_pedazen.rotate(v, torch.tensor([0, 5]), 4, 100.0)
    assert torch.equal(out[0], v[0]) and torch.equal(out[..., 4:], v[..., 4:])
    a = 5 * 100.0 ** (-2 / 4)
    assert abs(float(out[1, 0, 1]) - (8 * math.cos(a) - 10 * math.sin(a))) < 1e-9
    assert abs(float(out[1, 0, 3]) - (10 * math.cos(a) + 8 * math.sin(a))) < 1e-9
    # the router: softmax over all, the best groups only, the chosen scores normalised
    r = {"top": 2, "groups": {"count": 3, "keep": 2}}
    logits = torch.log(torch.tensor([[0.05, 0.30, 0.25, 0.02, 0.20, 0.18]], dtype=torch.float64))
    choice, weight = plain_pedazen.route(torch.eye(1, dtype=torch.float64), logits.T.contiguous(), r)
    # groups (0.05, 0.30), (0.25, 0.02), (0.20, 0.18): the best two are the first two, so 0.20 cannot be chosen
    assert choice.tolist() == [[1, 2]] and torch.allclose(weight, torch.tensor([[0.30 / 0.55, 0.25 / 0.55]], dtype=torch.float64))
    # the expert: the square of relu, no gate
    w = {"e.up": torch.tensor([[1.0], [-1.0]], dtype=torch.float64), "e.down": torch.tensor([[1.0, 10.0]], dtype=torch.float64)}
    assert plain_pedazen.expert(torch.tensor([[3.0]], dtype=torch.float64), w, "e.").tolist() == [[9.0]]
    assert plain_pedazen.expert(torch.tensor([[-2.0]], dtype=torch.float64), w, "e.").tolist() == [[40.0]]
    # lightning attention: two tokens, one head of size one; S1 = k1 v1, S2 = d S1 + k2 v2, o = S q
    m = {"heads": 1, "dim": 1, "vdim": 1, "decay": [0.5]}
    one = torch.ones(1, 1, dtype=torch.float64)
    lw = {"q": one, "k": one, "v": one, "g": 0 * one, "o": one, "norm": torch.ones(1, dtype=torch.float64)}
    h = torch.tensor([[1.0], [2.0]], dtype=torch.float64)
    s = lambda z: z / (1 + math.exp(-z))
    o1 = s(1.0) * s(1.0) * s(1.0)
    o2 = (0.5 * s(1.0) * s(1.0) + s(2.0) * s(2.0)) * s(2.0)
    got = plain_pedazen.lightning_mixer(h, lw, "", m, 0.0)
    # one element per row: the RMS norm leaves its sign, the gate sigmoid(0) halves it
    assert torch.allclose(got, torch.tensor([[0.5 * o1 / abs(o1)], [0.5 * o2 / abs(o2)]], dtype=torch.float64))
    # the recurrent block's first token has no special case: S1 = sqrt(1 - a^2) i u from S0 = 0
    rm = {"width": 1, "blocks": 1, "conv": 2}
    rw = {"y": one, "y.b": torch.zeros(1, dtype=torch.float64), "x": one, "x.b": torch.tensor([0.5], dtype=torch.float64),
          "conv": torch.tensor([[2.0, 3.0]], dtype=torch.float64), "conv.b": torch.tensor([0.25], dtype=torch.float64),
          "ra": one.view(1, 1, 1), "ra.b": torch.zeros(1, 1, dtype=torch.float64), "ri": one.view(1, 1, 1),
          "ri.b": torch.zeros(1, 1, dtype=torch.float64), "lam": torch.tensor([0.3], dtype=torch.float64), "o": one}
    out = plain_pedazen.recurrent_block(torch.tensor([[1.0]], dtype=torch.float64), rw, "", rm)
    u = 0.25 + 3.0 * 1.5                                       # the last tap is the current token's; zeros before the start
    sig = 1 / (1 + math.exp(-u))
    a = math.exp(-8 * sig * math.log1p(math.exp(0.3)))
    y = 0.5 * 1.0 * (1 + math.tanh(math.sqrt(2 / math.pi) * (1.0 + 0.044715)))
    assert abs(float(out) - math.sqrt(1 - a * a) * sig * u * y) < 1e-12
    # a sink takes weight from the keys and gives it to nothing: two equal keys and a sink of equal score
    am = {"heads": 1, "kv_heads": 1, "dim": 2, "vdim": 1, "rot": {"dims": 0, "base": 10.0}, "mask": {"size": 8}, "softcap": 1e6,
          "scale": 1.0}
    aw = {"q": torch.zeros(2, 1, dtype=torch.float64), "k": torch.zeros(2, 1, dtype=torch.float64), "v": one,
          "q.norm": torch.ones(2, dtype=torch.float64), "k.norm": torch.ones(2, dtype=torch.float64),
          "sink": torch.zeros(1, dtype=torch.float64), "o": one}
    out = plain_pedazen.chunked_sink_attention(torch.tensor([[3.0], [6.0]], dtype=torch.float64), aw, "", am, 1e-6)
    assert torch.allclose(out, torch.tensor([[3.0 / 2], [(3.0 + 6.0) / 3]], dtype=torch.float64))


def test_trace_replay_of_a_pedazen_folder(tmp_path):
    folder = cases.write_folder(str(tmp_path / "m"), cases.ODD, seed=5)
    cfg, w = cases.read_folder(folder)
    toks = helpers.random_tokens(cfg["vocab"], 15, 9)
    ref = _plain(cfg, w, toks)
    lines = [{"step": 0, "entries": [{"id": "a", "tokens": toks[:9], "want": [0, 8]}], "end": []},
             {"step": 1, "entries": [{"id": "a", "tokens": toks[9:11], "want": []}], "end": []},
             {"step": 2, "entries": [{"id": "a", "tokens": toks[11:], "want": [3]}], "end": ["a"]}]
    log = io.StringIO()
    run_trace(folder, "float32", str(tmp_path / "out"), 64, [json.dumps(l) for l in lines], log=log, device="cpu",
              kernels=TorchKernels(), page_size=16)
    assert log.getvalue().split() == ["done", "0", "done", "1", "done", "2"]
    s0 = np.fromfile(tmp_path / "out" / "0.f32", dtype="<f4").reshape(2, cfg["vocab"])
    s2 = np.fromfile(tmp_path / "out" / "2.f32", dtype="<f4").reshape(1, cfg["vocab"])
    scale = float(ref.abs().max())
    assert np.abs(s0 - ref[[0, 8]].numpy()).max() < 2e-5 * scale and np.abs(s2 - ref[[14]].numpy()).max() < 2e-5 * scale
    assert not (tmp_path / "out" / "1.f32").exists()


def test_greedy_generation_through_the_scheduler_under_page_pressure(tmp_path):
    from tt_transformers_b200.engine.llm import from_pretrained

    folder = cases.write_folder(str(tmp_path / "g"), cases.PLAIN, seed=7)
    cfg, w = cases.read_folder(folder)
    prompts = [helpers.random_tokens(cfg["vocab"], n, 80 + n) for n in (4, 13, 21)]

    def plain_greedy(prompt, new):
        toks = list(prompt)
        for _ in range(new):
            toks.append(int(_plain(cfg, w, toks)[-1].argmax()))
        return toks[len(prompt):]

    expect = [plain_greedy(p, 6) for p in prompts]
    # 7 pages of 8 tokens for requests that end at 10, 19 and 27 tokens: they cannot all stay, one gives way and is
    # recomputed from a zeroed state
    llm = from_pretrained(folder, dtype="float32", page_size=8, num_pages=7, max_batch_size=3, max_seq_len=64,
                          max_step_tokens=16, max_chunk_tokens=8, device="cpu", kernels=TorchKernels())
    assert llm.generate(prompts, max_new_tokens=6) == expect
    llm.engine.cache.audit()
    assert llm.engine.cache.free_pages() == 7
