"""The Bozavik decoder's configuration, read from its own config.json keys.

Top level: `architecture` ("Bozavik"), `vocab`, `width`, `residual_mult`, `norm.eps`, `embedding.scale` and
`layers`, a list whose entries give `type` (which mixer), `mixer` (its sizes and constants) and `mlp` (the
feed-forward, or null for a layer without one). Every size and constant comes from there; nothing is assumed
to be equal between layers.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

from .base import ConfigError, require, take

MIXER_TYPES = ("latent_attention", "latent_attention_2")


@dataclass(frozen=True)
class LatentMixerConfig:
    heads: int
    dim: int                 # unrotated query/key elements per head
    vdim: int                # value elements per head
    q_rank: int
    kv_rank: int
    scale: float
    rot_dim: int = 0         # rotated query/key elements per head (the key's are shared by all heads)
    rot_base: float = 0.0
    rot_dims: int = 0        # how many of the rotated part's elements the rotation covers


@dataclass(frozen=True)
class RoutedMlpConfig:
    experts: int
    top: int
    inter: int
    limit: float
    shared_inter: Optional[int] = None
    shared_limit: Optional[float] = None


@dataclass(frozen=True)
class BozavikLayer:
    type: str
    mixer: LatentMixerConfig
    mlp: Optional[RoutedMlpConfig]


@dataclass(frozen=True)
class BozavikConfig:
    architecture: str
    vocab: int
    width: int
    residual_mult: float
    norm_eps: float
    embedding_scale: float
    layers: Tuple[BozavikLayer, ...]

    # what the engine's entry points ask of any configuration
    eos_token_ids: tuple = ()
    bos_token_id: Optional[int] = None

    @property
    def vocab_size(self) -> int:
        return self.vocab

    @classmethod
    def from_dict(cls, data: dict) -> "BozavikConfig":
        norm = data.get("norm")
        require(isinstance(norm, dict), "config.json: 'norm' must be an object holding 'eps'")
        emb = data.get("embedding") or {}
        require(isinstance(emb, dict), "config.json: 'embedding' must be an object")
        raw_layers = data.get("layers")
        require(isinstance(raw_layers, list) and len(raw_layers) >= 1, "config.json: 'layers' must be a non-empty list")
        layers = tuple(_layer(i, entry) for i, entry in enumerate(raw_layers))
        cfg = cls(architecture=take(data, "architecture", str), vocab=take(data, "vocab", int),
                  width=take(data, "width", int), residual_mult=take(data, "residual_mult", float, 1.0),
                  norm_eps=take(norm, "eps", float, where="config.json: norm"),
                  embedding_scale=take(emb, "scale", float, 1.0, where="config.json: embedding"), layers=layers)
        require(cfg.vocab >= 1 and cfg.width >= 1, "config.json: 'vocab' and 'width' must be positive")
        return cfg


def _layer(i: int, entry) -> BozavikLayer:
    where = f"config.json: layers[{i}]"
    require(isinstance(entry, dict), f"{where} must be an object")
    kind = take(entry, "type", str, where=where)
    require(kind in MIXER_TYPES, f"{where}: type {kind!r} is not known; known: {list(MIXER_TYPES)}")
    m = entry.get("mixer")
    require(isinstance(m, dict), f"{where}: 'mixer' must be an object")
    mw = where + ".mixer"
    rot_dim = rot_dims = 0
    rot_base = 0.0
    if kind == "latent_attention_2":
        rot_dim = take(m, "rot_dim", int, where=mw)
        rot = m.get("rot")
        require(isinstance(rot, dict), f"{mw}: 'rot' must be an object holding 'base' and 'dims'")
        rot_base = take(rot, "base", float, where=mw + ".rot")
        rot_dims = take(rot, "dims", int, where=mw + ".rot")
        require(rot_dim >= 2 and 2 <= rot_dims <= rot_dim and rot_dims % 2 == 0,
                f"{mw}: rot.dims ({rot_dims}) must be even and at most rot_dim ({rot_dim})")
    mixer = LatentMixerConfig(heads=take(m, "heads", int, where=mw), dim=take(m, "dim", int, where=mw),
                              vdim=take(m, "vdim", int, where=mw), q_rank=take(m, "q_rank", int, where=mw),
                              kv_rank=take(m, "kv_rank", int, where=mw), scale=take(m, "scale", float, where=mw),
                              rot_dim=rot_dim, rot_base=rot_base, rot_dims=rot_dims)
    for key in ("heads", "dim", "vdim", "q_rank", "kv_rank"):
        require(getattr(mixer, key) >= 1, f"{mw}: '{key}' must be positive")
    mlp = None
    raw = entry.get("mlp")
    if raw is not None:
        lw = where + ".mlp"
        require(isinstance(raw, dict), f"{lw} must be an object or null")
        kind_mlp = take(raw, "kind", str, "moe", where=lw)
        if kind_mlp != "moe":
            raise ConfigError(f"{lw}: kind {kind_mlp!r} is not known; known: ['moe']")
        expert, router = raw.get("expert"), raw.get("router")
        require(isinstance(expert, dict) and isinstance(router, dict), f"{lw}: 'expert' and 'router' must be objects")
        shared = raw.get("shared")
        require(shared is None or isinstance(shared, dict), f"{lw}: 'shared' must be an object or null")
        mlp = RoutedMlpConfig(experts=take(router, "experts", int, where=lw + ".router"),
                              top=take(router, "top", int, where=lw + ".router"),
                              inter=take(expert, "ff", int, where=lw + ".expert"),
                              limit=take(expert, "limit", float, where=lw + ".expert"),
                              shared_inter=take(shared, "ff", int, where=lw + ".shared") if shared else None,
                              shared_limit=take(shared, "limit", float, where=lw + ".shared") if shared else None)
        require(1 <= mlp.top <= mlp.experts, f"{lw}.router: 'top' must lie between 1 and 'experts'")
    return BozavikLayer(type=kind, mixer=mixer, mlp=mlp)
