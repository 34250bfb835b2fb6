"""Train the liveSee surface-block classifier and render a chunk."""

from __future__ import annotations

import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE))
from _common import fit, write_metrics  # noqa: E402

from underhfs.functional import cross_entropy  # noqa: E402
from underhfs.optim import SGD  # noqa: E402
from underhfs.tensor import tensor  # noqa: E402

from live_world import LiveWorldModel, block_histogram, render_ascii, render_chunk, spawn_player, training_samples  # noqa: E402,E501

PROMPT = "glowing water ruins"


def train_model(prompt: str, steps: int) -> tuple[LiveWorldModel, list[float]]:
    feats, labels = training_samples(prompt)
    x, y = tensor(feats), tensor(labels)
    model = LiveWorldModel()
    losses = fit(model, SGD(model.parameters(), lr=0.05), lambda m: cross_entropy(m(x), y), steps)
    return model, losses


def run_smoke(*, steps: int = 18, write_artifacts: bool = False) -> dict:
    model, losses = train_model(PROMPT, steps)
    chunk = render_chunk(model, PROMPT, spawn_player(PROMPT), radius=4)
    report = {"project": "liveSee", "task": "minecraft_like_ai_live_world_generation_and_play", "prompt": PROMPT,
              "controls": "WASD + Q/E or arrow keys", "steps": steps, "initial_loss": losses[0],
              "final_loss": losses[-1], "mode": chunk["mode"], "player": chunk["player"],
              "ascii_view": render_ascii(chunk), "block_count": len(chunk["blocks"]),
              "block_histogram": block_histogram(chunk["blocks"])}
    if write_artifacts:
        write_metrics(HERE, report)
    return report


if __name__ == "__main__":
    print(json.dumps(run_smoke(write_artifacts=True), indent=2))
