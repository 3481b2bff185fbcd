"""The Bozavik decoder as a ModelSpec.

A scaled embedding table; per layer a `sandwich` block (layer norms with bias before and after each
sub-layer, a multiplier on what joins the float32 stream) around a latent-attention mixer and a routed
feed-forward; a final layer norm and an untied linear head. The two mixer types of the design are one
part kind with different options: `latent_attention` has no positions, a sink per head in the softmax's
denominator and one gate number per output element; `latent_attention_2` has a rotated part, an ordinary
softmax and one gate number per head. Tensor names: 'embed', 'l<i>.norm1' (+ '.b'), 'l<i>.norm1b',
'l<i>.norm2', 'l<i>.norm2b', 'l<i>.mix.*', 'l<i>.mlp.*', 'final.norm', 'head'.
"""

from __future__ import annotations

from ..config.bozavik import BozavikConfig
from ..parts import LayerCall, LayerSpec, ModelSpec, PartSpec


def load_config(data: dict) -> BozavikConfig:
    return BozavikConfig.from_dict(data)


def _norm(cfg: BozavikConfig, name: str) -> PartSpec:
    return PartSpec("layernorm", dict(width=cfg.width, eps=cfg.norm_eps, weight_name=name, bias_name=name + ".b"))


def model_spec(cfg: BozavikConfig) -> ModelSpec:
    layers = []
    for i, layer in enumerate(cfg.layers):
        p, m = f"l{i}.", layer.mixer
        second = layer.type == "latent_attention_2"
        parts = dict(
            norm1=_norm(cfg, p + "norm1"),
            mixer=PartSpec("latent_attention", dict(
                width=cfg.width, heads=m.heads, dim=m.dim, vdim=m.vdim, q_rank=m.q_rank, kv_rank=m.kv_rank,
                scale=m.scale, eps=cfg.norm_eps, prefix=p + "mix.", rot_dim=m.rot_dim,
                sink=not second, gate="head" if second else "element")),
            post1=_norm(cfg, p + "norm1b"))
        position = PartSpec("rotary", dict(rotary_dim=m.rot_dims, theta=m.rot_base, scaling=None)) if second else None
        if layer.mlp is None:
            layers.append(LayerSpec(block="sandwich_mixer_only", position=position,
                                    block_params=dict(residual_mult=cfg.residual_mult), **parts))
            continue
        f = layer.mlp
        parts.update(
            norm2=_norm(cfg, p + "norm2"),
            feed_forward=PartSpec("routed_experts", dict(
                width=cfg.width, experts=f.experts, top=f.top, inter=f.inter, limit=f.limit, prefix=p + "mlp.",
                shared_inter=f.shared_inter, shared_limit=f.shared_limit)),
            post2=_norm(cfg, p + "norm2b"))
        layers.append(LayerSpec(block="sandwich", position=position, block_params=dict(residual_mult=cfg.residual_mult),
                                **parts))
    return ModelSpec(
        vocab_size=cfg.vocab, width=cfg.width,
        embedding=PartSpec("table", dict(vocab=cfg.vocab, width=cfg.width, weight_name="embed", scale=cfg.embedding_scale)),
        layers=tuple(layers), order=tuple(LayerCall(i) for i in range(len(layers))),
        final_norm=_norm(cfg, "final.norm"),
        head=PartSpec("linear", dict(vocab=cfg.vocab, width=cfg.width, weight_name="head")),
    )


def ignorable(cfg: BozavikConfig, name: str) -> bool:
    # a layer without a feed-forward may still carry the norms around one
    for i, layer in enumerate(cfg.layers):
        if layer.mlp is None and name.startswith((f"l{i}.norm2", f"l{i}.mlp.")):
            return True
    return False
