"""The Pedazen decoder as a ModelSpec.

A scaled embedding table; per layer a `parallel` block (one RMS norm with a 1 + w weight whose output feeds
both the mixer and the feed-forward; both outputs join the float32 stream together) around a
`lightning_attention` mixer or a `mixer_pair` of `sink_attention` and `gated_recurrence`, and a `gated_mlp`
(tanh-GELU) or `grouped_experts` feed-forward; a final norm of the same kind and a head tied to the embedding
table. Looped layers are named several times in the layer order, each call with a cache unit of its own;
a `pass_entry` stream step stands before the first layer of every pass. Tensor names: 'embed', 'loop.step',
'l<i>.norm1', 'l<i>.mix.*', 'l<i>.mlp.*', 'final.norm'.
"""

from __future__ import annotations

from ..config.pedazen import PedazenConfig
from ..parts import LayerCall, LayerSpec, ModelSpec, PartSpec


def load_config(data: dict) -> PedazenConfig:
    return PedazenConfig.from_dict(data)


def _norm(cfg: PedazenConfig, name: str) -> PartSpec:
    return PartSpec("rmsnorm", dict(width=cfg.width, eps=cfg.norm_eps, weight_name=name, unit_offset=True))


def _feed_forward(cfg: PedazenConfig, f, prefix: str) -> PartSpec:
    if f.kind == "dense":
        return PartSpec("gated_mlp", dict(width=cfg.width, inter=f.inter, prefix=prefix, activation="gelu_tanh",
                                          names=("gate", "up", "down")))
    return PartSpec("grouped_experts", dict(width=cfg.width, experts=f.experts, top=f.top, inter=f.inter, prefix=prefix,
                                            groups=f.groups, keep=f.keep, activation="relu2"))


def model_spec(cfg: PedazenConfig) -> ModelSpec:
    layers = []
    for i, layer in enumerate(cfg.layers):
        p, m = f"l{i}.", layer.mixer
        position = None
        if layer.type == "lightning":
            mixer = PartSpec("lightning_attention", dict(width=cfg.width, heads=m.heads, dim=m.dim, vdim=m.vdim,
                                                         decay=m.decay, eps=cfg.norm_eps, prefix=p + "mix."))
        else:
            a, r = m.left, m.right
            left = PartSpec("sink_attention", dict(
                width=cfg.width, heads=a.heads, kv_heads=a.kv_heads, dim=a.dim, vdim=a.vdim, scale=a.scale,
                eps=cfg.norm_eps, prefix=p + "mix.left.", softcap=a.softcap, chunk=a.chunk, sink=True, qk_norm=True))
            right = PartSpec("gated_recurrence", dict(width=cfg.width, channels=r.channels, blocks=r.blocks, taps=r.taps,
                                                      prefix=p + "mix.right."))
            mixer = PartSpec("mixer_pair", dict(width=cfg.width, eps=cfg.norm_eps, left=left, right=right,
                                                left_norm=p + "mix.left.out", right_norm=p + "mix.right.out"))
            if a.rot_dims:
                position = PartSpec("rotary", dict(rotary_dim=a.rot_dims, theta=a.rot_base, scaling=None))
        parts = dict(norm1=_norm(cfg, p + "norm1"), mixer=mixer)
        if layer.mlp is None:
            layers.append(LayerSpec(block="parallel_mixer_only", position=position, **parts))
        else:
            layers.append(LayerSpec(block="parallel", position=position,
                                    feed_forward=_feed_forward(cfg, layer.mlp, p + "mlp."), **parts))
    n = len(layers)
    order, steps = [], []
    if cfg.loop_times:
        order += [LayerCall(i) for i in range(cfg.loop_start)]
        for t in range(cfg.loop_times):
            steps.append((len(order), PartSpec("pass_entry", dict(width=cfg.width, table_name="loop.step",
                                                                  rows=cfg.loop_times, row=t, add_embedding=t > 0))))
            order += [LayerCall(i) for i in range(cfg.loop_start, cfg.loop_stop)]
        order += [LayerCall(i) for i in range(cfg.loop_stop, n)]
    else:
        order = [LayerCall(i) for i in range(n)]
    return ModelSpec(
        vocab_size=cfg.vocab, width=cfg.width,
        embedding=PartSpec("table", dict(vocab=cfg.vocab, width=cfg.width, weight_name="embed", scale=cfg.embedding_scale)),
        layers=tuple(layers), order=tuple(order), stream_steps=tuple(steps),
        final_norm=_norm(cfg, "final.norm"),
        head=PartSpec("linear", dict(vocab=cfg.vocab, width=cfg.width, weight_name=None)),
    )


def ignorable(cfg: PedazenConfig, name: str) -> bool:
    return False
