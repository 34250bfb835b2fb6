"""3x3 gridworld imitation: (agent, goal) positions -> action logits, CE + SGD."""

from __future__ import annotations

import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from _common import fit, write_metrics  # noqa: E402

from underhfs.functional import cross_entropy  # noqa: E402
from underhfs.nn import Linear, ReLU, Sequential  # noqa: E402
from underhfs.optim import SGD  # noqa: E402
from underhfs.tensor import tensor  # noqa: E402

ACTIONS = ["up", "down", "left", "right"]
GOAL = (2, 2)


def expert_action(x: int, y: int) -> str:
    if x < GOAL[0]:
        return "right"
    if y < GOAL[1]:
        return "down"
    return "up"


def gridworld_states():
    cells = [(x, y) for y in range(3) for x in range(3)]
    states = [[x / 2.0, y / 2.0, GOAL[0] / 2.0, GOAL[1] / 2.0] for x, y in cells]
    labels = [ACTIONS.index(expert_action(x, y)) for x, y in cells]
    return states, labels


def build_model() -> Sequential:
    return Sequential(Linear(4, 8), ReLU(), Linear(8, len(ACTIONS)))


def run_smoke(*, steps: int = 16, write_artifacts: bool = False) -> dict:
    states, labels = gridworld_states()
    x, y = tensor(states), tensor(labels)
    model = build_model()
    losses = fit(model, SGD(model.parameters(), lr=0.08), lambda m: cross_entropy(m(x), y), steps)
    rows = model(x).tolist()
    report = {"project": "progamer_rl", "environment": "3x3 gridworld imitation seed", "steps": steps,
              "initial_loss": losses[0], "final_loss": losses[-1],
              "policy": [ACTIONS[r.index(max(r))] for r in rows], "oracle": [ACTIONS[i] for i in labels]}
    if write_artifacts:
        write_metrics(Path(__file__).resolve().parent, report)
    return report


if __name__ == "__main__":
    print(json.dumps(run_smoke(write_artifacts=True), indent=2))
