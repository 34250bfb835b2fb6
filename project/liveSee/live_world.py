"""liveSee: a prompt-conditioned voxel world whose surface blocks come from a
small classifier, with WASD/QE movement and chunk rendering.

Terrain height is an analytic sin/cos field of the prompt seed; below the
surface there are two dirt layers over stone; the surface block (grass,
stone, water, glowstone, ruin) is predicted by ``LiveWorldModel``
(MLP 10-18-7) trained on rule-generated labels.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Iterable

from underhfs.nn import Linear, ReLU, Sequential
from underhfs.tensor import Tensor, tensor

BLOCKS = {
    0: {"name": "air", "color": "#87c8ff", "solid": False},
    1: {"name": "grass", "color": "#55aa55", "solid": True},
    2: {"name": "dirt", "color": "#8b5a2b", "solid": True},
    3: {"name": "stone", "color": "#8c8c8c", "solid": True},
    4: {"name": "water", "color": "#3188d4", "solid": False},
    5: {"name": "glowstone", "color": "#f2c94c", "solid": True},
    6: {"name": "ruin", "color": "#5d6466", "solid": True},
}
AIR, GRASS, DIRT, STONE, WATER, GLOW, RUIN = range(7)


@dataclass(frozen=True)
class Player:
    x: float = 0.0
    y: float = 4.0
    z: float = 0.0
    yaw: float = 0.0


def _has(prompt: str, *words: str) -> bool:
    p = prompt.lower()
    return any(w in p for w in words)


def prompt_seed(prompt: str) -> int:
    return sum(i * b for i, b in enumerate(prompt.encode("utf-8"), start=1)) % 7919


def height_at(prompt: str, x: int, z: int) -> int:
    s = prompt_seed(prompt)
    wave = math.sin((x + s % 23) * 0.45) + math.cos((z - s % 17) * 0.38)
    lift = 2 if _has(prompt, "mountain", "cliff") else 0
    return max(1, min(8, 3 + int(round(wave + lift))))


def world_features(prompt: str, x: int, y: int, z: int) -> Tensor:
    s = prompt_seed(prompt)
    return tensor([[
        x / 16.0, y / 8.0, z / 16.0, math.sin(x * 0.37), math.cos(z * 0.41), math.sin((x + z) * 0.19),
        (s % 31) / 15.0 - 1.0, float(_has(prompt, "water", "ocean")), float(_has(prompt, "ruin", "city")),
        float(_has(prompt, "glow", "magic")),
    ]])


def target_surface_block(prompt: str, x: int, z: int) -> int:
    s = prompt_seed(prompt)
    noise = int(abs(math.sin((x * 31 + z * 17 + s) * 0.13)) * 1000)
    h = height_at(prompt, x, z)
    if _has(prompt, "water", "ocean") and h <= 3 and noise % 5 < 3:
        return WATER
    if _has(prompt, "ruin", "city") and (x - z + noise) % 11 < 2:
        return RUIN
    if _has(prompt, "glow", "magic") and (x + 2 * z + noise) % 13 == 0:
        return GLOW
    return STONE if h >= 6 else GRASS


class LiveWorldModel:
    def __init__(self) -> None:
        self.net = Sequential(Linear(10, 18), ReLU(), Linear(18, len(BLOCKS)))

    def parameters(self):
        return self.net.parameters()

    def __call__(self, features: Tensor) -> Tensor:
        return self.net(features)

    def predict_surface_block(self, prompt: str, x: int, z: int) -> int:
        logits = self.net(world_features(prompt, x, height_at(prompt, x, z), z)).tolist()[0]
        best = max(range(1, len(logits)), key=lambda i: logits[i])
        return best if BLOCKS[best]["solid"] else GRASS


def block_at(model: LiveWorldModel, prompt: str, x: int, y: int, z: int) -> int:
    ground = height_at(prompt, x, z)
    if y > ground:
        return AIR
    if y == ground:
        return model.predict_surface_block(prompt, x, z)
    return DIRT if y >= ground - 2 else STONE


def training_samples(prompt: str, radius: int = 5) -> tuple[list[list[float]], list[int]]:
    feats, labels = [], []
    for z in range(-radius, radius + 1):
        for x in range(-radius, radius + 1):
            feats.append(world_features(prompt, x, height_at(prompt, x, z), z).tolist()[0])
            labels.append(target_surface_block(prompt, x, z))
    return feats, labels


def player_dict(p: Player) -> dict[str, float]:
    return {"x": p.x, "y": p.y, "z": p.z, "yaw": p.yaw}


def render_chunk(model: LiveWorldModel, prompt: str, player: Player, *, radius: int = 8) -> dict:
    cx, cz = math.floor(player.x), math.floor(player.z)
    blocks = []
    for z in range(cz - radius, cz + radius + 1):
        for x in range(cx - radius, cx + radius + 1):
            ground = height_at(prompt, x, z)
            for y in range(max(0, ground - 3), ground + 1):
                b = block_at(model, prompt, x, y, z)
                if b == AIR:
                    continue
                info = BLOCKS[b]
                blocks.append({"x": x, "y": y, "z": z, "block": b, "name": info["name"], "color": info["color"],
                               "solid": info["solid"]})
    return {"prompt": prompt, "mode": "minecraft_like_voxel_world", "player": player_dict(player), "radius": radius,
            "blocks": blocks, "legend": {str(k): v for k, v in BLOCKS.items()}}


def spawn_player(prompt: str) -> Player:
    return Player(0.0, float(height_at(prompt, 0, 0) + 2), 0.0, 0.0)


_TURN = {"q": -0.25, "arrowleft": -0.25, "e": 0.25, "arrowright": 0.25}


def move(player: Player, direction: str, prompt: str = "", *, step: float = 1.0) -> Player:
    d = direction.lower()
    if d in _TURN:
        return Player(player.x, player.y, player.z, player.yaw + _TURN[d])
    fwd = (math.sin(player.yaw), -math.cos(player.yaw))
    side = (math.cos(player.yaw), math.sin(player.yaw))
    vec = {"w": fwd, "s": (-fwd[0], -fwd[1]), "d": side, "a": (-side[0], -side[1])}.get(d)
    if vec is None:
        return player
    x, z = player.x + vec[0] * step, player.z + vec[1] * step
    y = float(height_at(prompt, math.floor(x), math.floor(z)) + 2) if prompt else player.y
    return Player(round(x, 4), y, round(z, 4), player.yaw)


def render_ascii(chunk: dict) -> str:
    """Top-down view: highest block initial per column, '@' at the player."""
    p = chunk["player"]
    px, pz = int(round(float(p["x"]))), int(round(float(p["z"])))
    r = int(chunk["radius"])
    top: dict[tuple[int, int], tuple[int, str]] = {}
    for b in chunk["blocks"]:
        key = (int(b["x"]), int(b["z"]))
        if key not in top or int(b["y"]) >= top[key][0]:
            top[key] = (int(b["y"]), str(b["name"])[0].upper())
    lines = []
    for z in range(pz - r, pz + r + 1):
        lines.append("".join("@" if (x, z) == (px, pz) else top.get((x, z), (0, "."))[1]
                             for x in range(px - r, px + r + 1)))
    return "\n".join(lines)


def block_histogram(blocks: Iterable[dict]) -> dict[str, int]:
    hist: dict[str, int] = {}
    for b in blocks:
        hist[str(b["name"])] = hist.get(str(b["name"]), 0) + 1
    return hist
