"""The Pedazen decoder's configuration, read from its own config.json keys.

Top level: `architecture` ("Pedazen"), `vocab`, `width`, `norm.eps`, `embedding.scale`, `layers` and `loop`.
A layer gives `type` ("lightning": linear attention with a decay per head; "parallel": softmax attention and a
recurrent block side by side), `mixer` (its sizes and constants) and `mlp` (a dense or a routed feed-forward, or
null). `loop` {start, stop, times} runs layers start .. stop-1 `times` times in a row. Every size and constant
comes from there; nothing is assumed to be equal between layers.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

from .base import ConfigError, require, take

MIXER_TYPES = ("lightning", "parallel")


@dataclass(frozen=True)
class LightningConfig:
    heads: int
    dim: int
    vdim: int
    decay: Tuple[float, ...]


@dataclass(frozen=True)
class LeftConfig:
    heads: int
    kv_heads: int
    dim: int
    vdim: int
    scale: float
    softcap: Optional[float]
    chunk: Optional[int]
    rot_dims: int
    rot_base: float


@dataclass(frozen=True)
class RightConfig:
    channels: int
    blocks: int
    taps: int


@dataclass(frozen=True)
class ParallelConfig:
    left: LeftConfig
    right: RightConfig


@dataclass(frozen=True)
class MlpConfig:
    kind: str                    # "dense" or "moe"
    inter: int
    experts: int = 0
    top: int = 0
    groups: int = 1
    keep: int = 1


@dataclass(frozen=True)
class PedazenLayer:
    type: str
    mixer: object                # LightningConfig or ParallelConfig
    mlp: Optional[MlpConfig]


@dataclass(frozen=True)
class PedazenConfig:
    architecture: str
    vocab: int
    width: int
    norm_eps: float
    embedding_scale: float
    layers: Tuple[PedazenLayer, ...]
    loop_start: int = 0
    loop_stop: int = 0
    loop_times: int = 0          # 0: no loop (and no table of pass vectors)

    # what the engine's entry points ask of any configuration
    eos_token_ids: tuple = ()
    bos_token_id: Optional[int] = None

    @property
    def vocab_size(self) -> int:
        return self.vocab

    @classmethod
    def from_dict(cls, data: dict) -> "PedazenConfig":
        norm = data.get("norm")
        require(isinstance(norm, dict), "config.json: 'norm' must be an object holding 'eps'")
        emb = data.get("embedding") or {}
        require(isinstance(emb, dict), "config.json: 'embedding' must be an object")
        raw_layers = data.get("layers")
        require(isinstance(raw_layers, list) and len(raw_layers) >= 1, "config.json: 'layers' must be a non-empty list")
        layers = tuple(_layer(i, entry) for i, entry in enumerate(raw_layers))
        start = stop = times = 0
        loop = data.get("loop")
        if loop is not None:
            require(isinstance(loop, dict), "config.json: 'loop' must be an object or null")
            start, stop = take(loop, "start", int, where="config.json: loop"), take(loop, "stop", int, where="config.json: loop")
            times = take(loop, "times", int, where="config.json: loop")
            require(0 <= start < stop <= len(layers), f"config.json: loop: start {start} .. stop {stop} must name layers of the {len(layers)}")
            require(times >= 1, "config.json: loop: 'times' must be at least 1")
        cfg = cls(architecture=take(data, "architecture", str), vocab=take(data, "vocab", int),
                  width=take(data, "width", int), norm_eps=take(norm, "eps", float, where="config.json: norm"),
                  embedding_scale=take(emb, "scale", float, 1.0, where="config.json: embedding"), layers=layers,
                  loop_start=start, loop_stop=stop, loop_times=times)
        require(cfg.vocab >= 1 and cfg.width >= 1, "config.json: 'vocab' and 'width' must be positive")
        return cfg


def _positive(obj, keys, where):
    for key in keys:
        require(getattr(obj, key) >= 1, f"{where}: '{key}' must be positive")


def _lightning(m: dict, where: str) -> LightningConfig:
    decay = m.get("decay")
    require(isinstance(decay, list) and all(isinstance(d, (int, float)) and not isinstance(d, bool) for d in decay),
            f"{where}: 'decay' must be a list of numbers, one per head")
    cfg = LightningConfig(heads=take(m, "heads", int, where=where), dim=take(m, "dim", int, where=where),
                          vdim=take(m, "vdim", int, where=where), decay=tuple(float(d) for d in decay))
    _positive(cfg, ("heads", "dim", "vdim"), where)
    require(len(cfg.decay) == cfg.heads, f"{where}: {len(cfg.decay)} decays for {cfg.heads} heads")
    return cfg


def _left(m: dict, where: str) -> LeftConfig:
    rot, mask = m.get("rot"), m.get("mask")
    require(rot is None or isinstance(rot, dict), f"{where}: 'rot' must be an object holding 'base' and 'dims'")
    require(mask is None or isinstance(mask, dict), f"{where}: 'mask' must be an object holding 'size'")
    cfg = LeftConfig(heads=take(m, "heads", int, where=where), kv_heads=take(m, "kv_heads", int, where=where),
                     dim=take(m, "dim", int, where=where), vdim=take(m, "vdim", int, where=where),
                     scale=take(m, "scale", float, where=where), softcap=take(m, "softcap", float, None, where=where),
                     chunk=take(mask, "size", int, where=where + ".mask") if mask else None,
                     rot_dims=take(rot, "dims", int, where=where + ".rot") if rot else 0,
                     rot_base=take(rot, "base", float, where=where + ".rot") if rot else 0.0)
    _positive(cfg, ("heads", "kv_heads", "dim", "vdim"), where)
    require(cfg.heads % cfg.kv_heads == 0, f"{where}: 'heads' ({cfg.heads}) must be a multiple of 'kv_heads' ({cfg.kv_heads})")
    require(cfg.rot_dims % 2 == 0 and 0 <= cfg.rot_dims <= cfg.dim,
            f"{where}: rot.dims ({cfg.rot_dims}) must be even and at most 'dim' ({cfg.dim})")
    require(cfg.chunk is None or cfg.chunk >= 1, f"{where}: mask.size must be positive")
    require(cfg.softcap is None or cfg.softcap > 0, f"{where}: 'softcap' must be positive")
    return cfg


def _right(m: dict, where: str) -> RightConfig:
    cfg = RightConfig(channels=take(m, "width", int, where=where), blocks=take(m, "blocks", int, where=where),
                      taps=take(m, "conv", int, where=where))
    _positive(cfg, ("channels", "blocks", "taps"), where)
    require(cfg.channels % cfg.blocks == 0, f"{where}: 'width' ({cfg.channels}) must split into 'blocks' ({cfg.blocks}) equal parts")
    return cfg


def _mlp(raw, where: str) -> Optional[MlpConfig]:
    if raw is None:
        return None
    require(isinstance(raw, dict), f"{where} must be an object or null")
    kind = take(raw, "kind", str, where=where)
    if kind == "dense":
        cfg = MlpConfig(kind=kind, inter=take(raw, "ff", int, where=where))
        require(cfg.inter >= 1, f"{where}: 'ff' must be positive")
        return cfg
    if kind != "moe":
        raise ConfigError(f"{where}: kind {kind!r} is not known; known: ['dense', 'moe']")
    expert, router = raw.get("expert"), raw.get("router")
    require(isinstance(expert, dict) and isinstance(router, dict), f"{where}: 'expert' and 'router' must be objects")
    groups = router.get("groups")
    require(groups is None or isinstance(groups, dict), f"{where}.router: 'groups' must be an object holding 'count' and 'keep'")
    cfg = MlpConfig(kind=kind, inter=take(expert, "ff", int, where=where + ".expert"),
                    experts=take(router, "experts", int, where=where + ".router"),
                    top=take(router, "top", int, where=where + ".router"),
                    groups=take(groups, "count", int, where=where + ".router.groups") if groups else 1,
                    keep=take(groups, "keep", int, where=where + ".router.groups") if groups else 1)
    require(cfg.inter >= 1, f"{where}.expert: 'ff' must be positive")
    require(1 <= cfg.top <= cfg.experts, f"{where}.router: 'top' must lie between 1 and 'experts'")
    require(cfg.groups >= 1 and cfg.experts % cfg.groups == 0,
            f"{where}.router: 'experts' ({cfg.experts}) must split into groups.count ({cfg.groups}) equal groups")
    require(1 <= cfg.keep <= cfg.groups, f"{where}.router.groups: 'keep' must lie between 1 and 'count'")
    require(cfg.keep * (cfg.experts // cfg.groups) >= cfg.top,
            f"{where}.router: the experts of groups.keep groups are fewer than 'top'")
    return cfg


def _layer(i: int, entry) -> PedazenLayer:
    where = f"config.json: layers[{i}]"
    require(isinstance(entry, dict), f"{where} must be an object")
    kind = take(entry, "type", str, where=where)
    require(kind in MIXER_TYPES, f"{where}: type {kind!r} is not known; known: {list(MIXER_TYPES)}")
    m = entry.get("mixer")
    require(isinstance(m, dict), f"{where}: 'mixer' must be an object")
    if kind == "lightning":
        mixer = _lightning(m, where + ".mixer")
    else:
        left, right = m.get("left"), m.get("right")
        require(isinstance(left, dict) and isinstance(right, dict), f"{where}.mixer: 'left' and 'right' must be objects")
        mixer = ParallelConfig(left=_left(left, where + ".mixer.left"), right=_right(right, where + ".mixer.right"))
    return PedazenLayer(type=kind, mixer=mixer, mlp=_mlp(entry.get("mlp"), where + ".mlp"))
