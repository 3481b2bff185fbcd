"""Bozavik on the GPU: every kernel of the design against its plain twin, and the whole engine (step function,
cache, captured decode steps, scheduler and entry point) against the plain implementation."""

from types import SimpleNamespace

import pytest
import torch

import bozavik_cases as cases
import helpers
import plain_bozavik
from torch_kernels import TorchKernels
from tt_transformers_b200.config import EngineConfig
from tt_transformers_b200.engine.step import build_engine
from tt_transformers_b200.parts import LatentPages

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def kernels():
    from tt_transformers_b200.kernels import load_kernels
    return load_kernels(torch.device(DEV))


@pytest.fixture(scope="module")
def twin():
    return TorchKernels(DEV)


def _norm(width, seed, bias=True):
    g = torch.Generator().manual_seed(seed)
    return SimpleNamespace(weight=(1 + 0.3 * torch.randn(width, generator=g)).to(DEV),
                           bias=(0.5 * torch.randn(width, generator=g)).to(DEV) if bias else None, eps=1e-5)


def _close(got, ref, tol):
    assert got.shape == ref.shape
    err = float((got.float() - ref.float()).abs().max()) / max(float(ref.float().abs().max()), 1e-6)
    assert err < tol, err


# ---------------------------------------------------------------------------- layer norm around sub-layers
@pytest.mark.parametrize("width", [60, 128, 1000, 2056])
@pytest.mark.parametrize("delta_dtype", [None, torch.float32, torch.bfloat16])
def test_add_layernorm(kernels, twin, width, delta_dtype):
    g = torch.Generator().manual_seed(width)
    for after, norm in ((None, _norm(width, 1)), (_norm(width, 2), _norm(width, 3, bias=False)), (_norm(width, 4), None)):
        if delta_dtype is None and after is not None:
            continue
        x = (3 + 2 * torch.randn(5, width, generator=g)).to(DEV)        # a mean far from zero: the variance is about it
        delta = None if delta_dtype is None else torch.randn(5, width, generator=g).to(DEV, delta_dtype)
        x_ref = x.clone()
        ref = twin.add_layernorm(x_ref, delta, after, 0.5, norm, torch.float32)
        got = kernels.add_layernorm(x, delta, after, 0.5, norm, torch.float32)
        _close(x, x_ref, 1e-5)
        if norm is not None:
            _close(got, ref, 1e-5)


# ---------------------------------------------------------------------------- the latent cache and attention over it
def _latent_setup(segs, H, R, extra, rotary_dim, page, dtype, seed, shuffle_pages=True):
    """segs: [(cached tokens, new tokens)]. A cache filled for all positions below pos0 + n, on pages in a shuffled
    order; queries for the new tokens."""
    g = torch.Generator().manual_seed(seed)
    width = max(-(-(p + n) // page) for p, n in segs)
    total_pages = sum(-(-(p + n) // page) for p, n in segs)
    order = (torch.randperm(total_pages, generator=g) + 1).tolist() if shuffle_pages else list(range(1, total_pages + 1))
    rows = torch.full((total_pages + 1, page, R + extra), float("nan"))
    table = torch.zeros(len(segs), width, dtype=torch.int32)
    at = 0
    for r, (p, n) in enumerate(segs):
        for i in range(-(-(p + n) // page)):
            table[r, i] = order[at]
            fill = min(page, p + n - i * page)
            rows[order[at], :fill] = torch.randn(fill, R + extra, generator=g)
            at += 1
    T = sum(n for _, n in segs)
    lens = [n for _, n in segs]
    pos0 = [p for p, _ in segs]
    positions = torch.cat([torch.arange(p, p + n) for p, n in segs]).to(torch.int32)
    seg_of = torch.cat([torch.full((n,), r) for r, (_, n) in enumerate(segs)]).to(torch.int32)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    batch = SimpleNamespace(positions=positions.to(DEV), seg_of_token=seg_of.to(DEV), cu_seqlens=cu.to(DEV),
                            seg_pos0=torch.tensor(pos0, dtype=torch.int32, device=DEV), seg_lens=lens, seg_pos0_list=pos0,
                            num_segments=len(segs), max_seg_len=max(lens), max_context=max(p + n for p, n in segs),
                            num_tokens=T)
    view = LatentPages(R, extra).view({"rows": rows.to(DEV, dtype)}, block_table=table.to(DEV), page_size=page)
    q_lat = (torch.randn(T, H, R, generator=g) * R ** -0.5).to(DEV, dtype)
    q_rot = (torch.randn(T, H, extra, generator=g) * 0.3).to(DEV, dtype) if extra else None
    inv_freq = (1.0 / 1000.0 ** (torch.arange(0, rotary_dim, 2).float() / rotary_dim)).to(DEV) if extra else None
    sinks = (torch.randn(H, generator=g) * 2).to(DEV)
    return batch, view, q_lat, q_rot, inv_freq, sinks


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-5), (torch.bfloat16, 2e-2)])
@pytest.mark.parametrize("H,R,extra,rotary_dim,page", [(7, 80, 0, 0, 16), (4, 112, 48, 32, 16), (5, 40, 12, 8, 4),
                                                       (1, 20, 0, 0, 8), (70, 32, 16, 16, 16), (3, 272, 16, 16, 32), (2, 528, 0, 0, 16)])
def test_latent_attention_against_its_twin(kernels, twin, dtype, tol, H, R, extra, rotary_dim, page):
    # a prompt portion beside cached tokens, decoded tokens at short and long contexts, a first token, and
    # portions that end just before, on and just after the edges of pages and of key tiles
    segs = [(0, 70), (129, 1), (63, 2), (64, 1), (0, 1), (300, 1), (127, 3), (page - 1, 2), (15, 40)]
    batch, view, q_lat, q_rot, inv_freq, sinks = _latent_setup(segs, H, R, extra, rotary_dim, page, dtype, seed=H * R)
    for use_sinks in (sinks, None):
        ref = twin.latent_attention(q_lat, q_rot, batch, view, 0.2, use_sinks, inv_freq, rotary_dim)
        got = kernels.latent_attention(q_lat, q_rot, batch, view, 0.2, use_sinks, inv_freq, rotary_dim)
        assert not torch.isnan(got.float()).any()               # nothing came from a row that was never written
        _close(got, ref, tol)
        if dtype == torch.bfloat16:                              # the float32-arithmetic kernel on the same storage
            kernels.use_mma_latent_attention = False
            try:
                _close(kernels.latent_attention(q_lat, q_rot, batch, view, 0.2, use_sinks, inv_freq, rotary_dim), ref, tol)
            finally:
                kernels.use_mma_latent_attention = True
    # the mixer's end in one call (key splits merged, W_uv per head, gate), with few tokens and with many
    g = torch.Generator().manual_seed(3)
    for V, gate_cols in ((16, H), (24, H * 24), (8, 0)):
        w_uv = (torch.randn(H, V, R, generator=g) * R ** -0.5).to(DEV, dtype)
        gate = torch.randn(batch.num_tokens, gate_cols, generator=g).to(DEV) if gate_cols else None
        for rows_limit in (1000, 0):
            kernels.LATENT_OUT_ROWS, keep = rows_limit, kernels.LATENT_OUT_ROWS
            try:
                got_out = kernels.latent_attention_out(q_lat, q_rot, batch, view, 0.2, sinks, inv_freq, rotary_dim, w_uv, gate)
            finally:
                kernels.LATENT_OUT_ROWS = keep
            _close(got_out, twin.latent_attention_out(q_lat, q_rot, batch, view, 0.2, sinks, inv_freq, rotary_dim, w_uv, gate), tol)
    with_sink = kernels.latent_attention(q_lat, q_rot, batch, view, 0.2, sinks + 3.0, inv_freq, rotary_dim)
    assert float((with_sink.float() - got.float()).abs().max()) > 0.05       # a sink that is left out shows


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("far", [0, 15, 16, 63, 64, 127, 128, 700, 1022, 1023])
def test_one_key_far_away_carries_the_weight(kernels, dtype, far):
    """One query (a decoded token at position 1023, then the last token of a portion of 5) whose score with the key
    at `far` stands out: the output must be that key's latent, wherever it lies (first token, page and tile edges,
    the query's own position)."""
    H, R, extra, page = 4, 64, 16, 16
    for segs in ([(1023, 1)], [(1019, 5)]):
        batch, view, q_lat, q_rot, inv_freq, _ = _latent_setup(segs, H, R, extra, 16, page, dtype, seed=far, shuffle_pages=True)
        table = view.block_table[0]
        target = view.rows[table[far // page].long(), far % page, :R].float()
        q_lat[-1] = (target / target.norm() * 40.0).to(dtype)            # score with the key at `far`: about 40 |c| = 320
        q_rot.zero_()
        got = kernels.latent_attention(q_lat, q_rot, batch, view, 1.0, None, inv_freq, 16)[-1].float()
        for h in range(H):
            assert float((got[h] - target).abs().max()) < 0.05, (segs, h)
        # the same through the mixer's fused end (key splits merged inside it), W_uv the identity
        eye = torch.eye(R, device=DEV, dtype=dtype).expand(H, R, R).contiguous()
        fused = kernels.latent_attention_out(q_lat, q_rot, batch, view, 1.0, None, inv_freq, 16, eye, None)[-1].float().view(H, R)
        for h in range(H):
            assert float((fused[h] - target).abs().max()) < 0.05, (segs, h, "fused")


def test_a_window_edge_in_the_general_kernel(kernels, twin):
    """A window is a parameter of the cache request; only the float32-arithmetic kernel takes one. Keys just inside
    and just outside it, in a portion and in decoding."""
    H, R, page = 3, 32, 8
    for window in (1, 5, 64, 65):
        segs = [(0, 80), (100, 1), (window, 1), (max(window - 1, 0), 2)]
        batch, view, q_lat, _, _, sinks = _latent_setup(segs, H, R, 0, 0, page, torch.float32, seed=window)
        view.window = window
        q_lat[:] = q_lat * 8                                                # sharp weights: one key more or less shows
        got = kernels.latent_attention(q_lat, None, batch, view, 1.0, sinks, None, 0)
        # the twin has no window: build the reference from the same twin on a cache whose older rows are pushed away
        ref = torch.empty_like(got)
        start = 0
        for r, (p, n) in enumerate(segs):
            for i in range(n):
                pos = p + i
                keys = torch.stack([view.rows[view.block_table[r, j // page].long(), j % page] for j in range(max(0, pos - window + 1), pos + 1)])
                s = torch.einsum("hr,sr->hs", q_lat[start + i], keys)
                full = torch.cat([s, sinks[:, None]], dim=1)
                wts = torch.softmax(full, dim=1)[:, :-1]
                ref[start + i] = wts @ keys
            start += n
        _close(got, ref, 2e-5)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 1e-2)])
def test_latent_prepare_heads_linear_and_gate(kernels, twin, dtype, tol):
    g = torch.Generator().manual_seed(1)
    for q_rank, R, rot, rotary_dim, gate_cols in ((48, 64, 16, 16, 4), (28, 36, 0, 0, 20), (18, 22, 6, 4, 0)):
        segs = [(0, 9), (37, 1), (5, 3)]
        batch, view, *_ = _latent_setup(segs, 2, R, rot, rotary_dim, 8, dtype, seed=R)
        view_ref = LatentPages(R, rot).view({"rows": view.rows.clone()}, block_table=view.block_table, page_size=8)
        T = batch.num_tokens
        down = (torch.randn(T, q_rank + R + rot + gate_cols, generator=g) * 2).to(DEV)
        qn, kn = (1 + 0.2 * torch.randn(q_rank, generator=g)).to(DEV), (1 + 0.2 * torch.randn(R, generator=g)).to(DEV)
        inv_freq = (1.0 / 500.0 ** (torch.arange(0, rotary_dim, 2).float() / rotary_dim)).to(DEV) if rot else None
        ref = twin.latent_prepare(down, batch, q_rank, R, rot, qn, kn, 1e-5, inv_freq, rotary_dim, view_ref, True, dtype)
        got = kernels.latent_prepare(down, batch, q_rank, R, rot, qn, kn, 1e-5, inv_freq, rotary_dim, view, True, dtype)
        _close(got, ref, tol)
        written = ~torch.isnan(view_ref.rows.float())
        assert torch.equal(written, ~torch.isnan(view.rows.float()))
        _close(torch.where(written, view.rows.float(), 0), torch.where(written, view_ref.rows.float(), 0), tol)
    for T in (1, 5, 40):                                    # per-head products on views with strides, few and many rows
        x = torch.randn(T, 3, 24 + 8, generator=g).to(DEV, dtype)[:, :, :24]
        w = torch.randn(3, 20, 24, generator=g).to(DEV, dtype)
        _close(kernels.heads_linear(x, w), twin.heads_linear(x, w), tol)
        out = kernels.heads_linear(x, w)
        for gate in (None, torch.randn(T, 3, generator=g).to(DEV), torch.randn(T, 60, generator=g).to(DEV)):
            _close(kernels.gate_heads(out, gate), twin.gate_heads(out, gate), tol)


# ---------------------------------------------------------------------------- the routed feed-forward
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-5), (torch.bfloat16, 2e-2)])
@pytest.mark.parametrize("T,width,E,top,inter", [(1, 64, 8, 2, 32), (7, 60, 5, 5, 20), (150, 128, 6, 3, 48), (40, 96, 1, 1, 72),
                                                 (600, 128, 5, 2, 72), (520, 320, 3, 2, 136)])
def test_router_and_experts_against_their_twins(kernels, twin, dtype, tol, T, width, E, top, inter):
    g = torch.Generator().manual_seed(T + E)
    x = torch.randn(T, width, generator=g).to(DEV, dtype)
    w_router = torch.randn(E + 1, width, generator=g).to(DEV)
    choice, weight, gate = kernels.route_top(x, w_router, E, top, True)
    c_ref, w_ref, g_ref = twin.route_top(x, w_router, E, top, True)
    assert torch.equal(choice, c_ref)
    _close(weight, w_ref, 1e-5)
    _close(gate, g_ref, 1e-5)
    assert torch.allclose(weight.sum(-1), torch.ones(T, device=DEV), atol=1e-5)
    w_gate_up = (torch.randn(E, 2 * inter, width, generator=g) * width ** -0.5 * 3).to(DEV, dtype)   # large enough to meet the limit
    w_down = (torch.randn(E, width, inter, generator=g) * inter ** -0.5).to(DEV, dtype)
    s_inter = 40
    shared = ((torch.randn(2 * s_inter, width, generator=g) * width ** -0.5 * 3).to(DEV, dtype),
              (torch.randn(width, s_inter, generator=g) * s_inter ** -0.5).to(DEV, dtype), 0.7)
    for shared_expert, shared_gate in ((shared, gate), (None, None)):
        got = kernels.routed_experts(x, choice, weight, w_gate_up, w_down, 1.5, 1.702, shared_expert, shared_gate)
        ref = twin.routed_experts(x, choice, weight, w_gate_up, w_down, 1.5, 1.702, shared_expert, shared_gate)
        assert got.dtype == torch.float32
        _close(got, ref, tol)
    gu = (torch.randn(T, 2 * inter, generator=g) * 3).to(DEV, dtype)
    _close(kernels.glu_clamped(gu, 1.5, 1.702), twin._glu_clamped(gu, 1.5, 1.702).to(dtype), tol)


def test_router_with_more_choices_than_a_warp_has_lanes(kernels, twin):
    g = torch.Generator().manual_seed(8)
    x = torch.randn(5, 48, generator=g).to(DEV)
    w = torch.randn(70, 48, generator=g).to(DEV)
    choice, weight, _ = kernels.route_top(x, w, 70, 40, False)
    c_ref, w_ref, _ = twin.route_top(x, w, 70, 40, False)
    assert torch.equal(choice, c_ref)
    _close(weight, w_ref, 1e-5)


def test_equal_router_logits_go_to_the_lower_index(kernels):
    x = torch.zeros(2, 16, device=DEV)
    x[1, 0] = 1.0
    w = torch.zeros(6, 16, device=DEV)
    w[4, 0] = w[2, 0] = 3.0                   # token 1: experts 2 and 4 tie for the lead, the rest tie at zero
    choice, weight, _ = kernels.route_top(x, w, 6, 3, False)
    assert choice.tolist() == [[0, 1, 2], [2, 4, 0]]
    assert torch.allclose(weight[0], torch.full((3,), 1 / 3, device=DEV))


def test_a_token_alone_and_in_a_crowd_gets_the_same_expert_output(kernels):
    g = torch.Generator().manual_seed(4)
    x = torch.randn(90, 64, generator=g).to(DEV, torch.bfloat16)
    w_router = torch.randn(8, 64, generator=g).to(DEV)
    w_gate_up = (torch.randn(8, 64, 64, generator=g) * 0.2).to(DEV, torch.bfloat16)
    w_down = (torch.randn(8, 64, 32, generator=g) * 0.2).to(DEV, torch.bfloat16)
    choice, weight, _ = kernels.route_top(x, w_router, 8, 2, False)
    crowd = kernels.routed_experts(x, choice, weight, w_gate_up, w_down, 2.0, 1.702, None, None)
    for t in (0, 33, 89):
        c1, w1, _ = kernels.route_top(x[t:t + 1], w_router, 8, 2, False)
        alone = kernels.routed_experts(x[t:t + 1], c1, w1, w_gate_up, w_down, 2.0, 1.702, None, None)
        _close(alone[0], crowd[t], 2e-2)


# ---------------------------------------------------------------------------- the whole model through the engine
@pytest.fixture(scope="module")
def folders(tmp_path_factory):
    root = tmp_path_factory.mktemp("bozavik")
    return {name: cases.write_folder(str(root / name), getattr(cases, name), seed=11) for name in ("ALIGNED", "ODD")}


@pytest.mark.parametrize("name", ["ALIGNED", "ODD"])
@pytest.mark.parametrize("dtype,tol", [("float32", 1e-4), ("bfloat16", 6e-2)])
def test_engine_matches_the_plain_implementation_however_the_requests_are_cut(folders, name, dtype, tol):
    cfg, w = cases.read_folder(folders[name])
    lengths = (150, 1, 23, 66, 97, 2)
    requests = {f"r{i}": helpers.random_tokens(cfg["vocab"], n, 30 + i) for i, n in enumerate(lengths)}
    ref = {rid: plain_bozavik.forward(cfg, w, toks) for rid, toks in requests.items()}
    for make_steps in (helpers.steps_whole, helpers.steps_decode_tail, helpers.steps_portions, helpers.steps_mixed):
        steps = make_steps(requests)
        pages = -(-helpers.max_live_tokens(requests, steps, rounding=8) // 8)
        engine = build_engine(folders[name], EngineConfig(dtype=dtype, page_size=8, num_pages=pages, max_batch_size=4,
                                                          max_seq_len=256, device=DEV))
        assert engine.graphs is not None                     # decode steps are replays of captured steps
        for g in engine.cache.groups:
            g.storage["rows"].fill_(float("nan"))
        got = helpers.run_steps(engine, steps)
        engine.cache.audit()
        assert engine.cache.free_pages() == pages
        for rid in ref:
            if dtype == "float32":
                assert helpers.relative_error(got[rid], ref[rid]) < tol, (make_steps.__name__, rid)
            else:
                # in bfloat16 a router's close call may go the other way for a token or two (top 1 of 7 experts):
                # nine rows in ten must agree, and the typical row closely
                scale = float(ref[rid].abs().max())
                rows = (got[rid] - ref[rid]).abs().amax(dim=-1) / scale
                assert float((rows < tol).float().mean()) >= 0.9 and float(rows.median()) < tol / 2, (make_steps.__name__, rid)
        engine.close()


@pytest.mark.parametrize("dtype,tol", [("float32", 1e-4), ("bfloat16", 6e-2)])
def test_a_long_prompt_whole_in_portions_and_decoded(folders, dtype, tol):
    """700 tokens: the expert products over groups of rows, attention over many key tiles, decoding at a long context."""
    cfg, w = cases.read_folder(folders["ALIGNED"])
    requests = {"long": helpers.random_tokens(cfg["vocab"], 700, 5), "other": helpers.random_tokens(cfg["vocab"], 90, 6)}
    ref = {rid: plain_bozavik.forward(cfg, w, toks) for rid, toks in requests.items()}
    for steps in (helpers.steps_whole(requests), helpers.steps_decode_tail(requests, 40),
                  helpers.steps_portions(requests, sizes=(130, 2, 257, 64, 3, 190)), helpers.steps_mixed(requests, decode_tail=20)):
        pages = -(-helpers.max_live_tokens(requests, steps, rounding=16) // 16)
        engine = build_engine(folders["ALIGNED"], EngineConfig(dtype=dtype, page_size=16, num_pages=pages, max_batch_size=2,
                                                               max_seq_len=1024, device=DEV))
        for g in engine.cache.groups:
            g.storage["rows"].fill_(float("nan"))
        got = helpers.run_steps(engine, steps)
        engine.cache.audit()
        for rid in ref:
            scale = float(ref[rid].abs().max())
            rows = (got[rid] - ref[rid]).abs().amax(dim=-1) / scale
            if dtype == "float32":
                assert float(rows.max()) < tol, rid
            else:
                assert float((rows < tol).float().mean()) >= 0.9 and float(rows.median()) < tol / 2, rid
        engine.close()


def test_residual_stream_after_every_layer(folders):
    """Layer by layer in float32: the model cut to its first k layers, then the final norm and head of the plain
    implementation applied to the plain residual stream at that depth."""
    cfg, w = cases.read_folder(folders["ALIGNED"])
    toks = helpers.random_tokens(cfg["vocab"], 21, 2)
    _, layers = plain_bozavik.forward(cfg, w, toks, keep_layers=True)
    for k in range(1, len(cfg["layers"]) + 1):
        engine = build_engine(folders["ALIGNED"], EngineConfig(dtype="float32", page_size=8, max_batch_size=1, max_seq_len=32,
                                                               device=DEV), n_layers=k)
        got = helpers.run_steps(engine, helpers.steps_whole({"a": toks}))["a"]
        ref = plain_bozavik.layer_norm(layers[k - 1], w["final.norm"], w["final.norm.b"], cfg["norm"]["eps"]) @ w["head"].T
        assert helpers.relative_error(got, ref) < 1e-4, k
        engine.close()


def test_long_decoding_and_greedy_generation_through_the_entry_point(folders):
    from tt_transformers_b200 import from_pretrained

    cfg, w = cases.read_folder(folders["ALIGNED"])
    prompts = [helpers.random_tokens(cfg["vocab"], n, 50 + n) for n in (5, 40, 17)]
    new = 70

    def plain_greedy(prompt):
        toks = list(prompt)
        for _ in range(new):
            toks.append(int(plain_bozavik.forward(cfg, w, toks)[-1].argmax()))
        return toks[len(prompt):]

    expect = [plain_greedy(p) for p in prompts]
    llm = from_pretrained(folders["ALIGNED"], dtype="float32", page_size=8, num_pages=60, max_batch_size=3, max_seq_len=128,
                          max_step_tokens=32, max_chunk_tokens=16, device=DEV)
    assert llm.generate(prompts, max_new_tokens=new) == expect
    # a second round on the pages and slots that the first gave back
    assert llm.generate(prompts[::-1], max_new_tokens=new) == expect[::-1]
    llm.engine.cache.audit()
    llm.cleanup()
