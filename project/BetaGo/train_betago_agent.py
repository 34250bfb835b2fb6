"""BetaGo: a 9x9 Go policy/value network trained on labelled positions.

Model (same shape as the reference agent, project/BetaGo/train_betago_agent.py
of the reference): trunk Linear(324,32)-ReLU-Linear(32,16)-ReLU, policy head
-> 82 moves (81 points + pass), value head -> 1.  Loss = cross-entropy(policy)
+ 0.35 * MSE(value), AdamW lr 0.015 wd 1e-4, 60 steps of batch 8.  Input
planes: own stones, opponent stones, legal moves, side to move.

Two datasets:

* ``task="reference"`` (default): the reference project's supervision task,
  restated here so the two runtimes train on identical data and their metrics
  compare -- positions from its seeded scatter generator or its eight
  strategy motifs (capture, defend-atari, connect, corner framework, side
  extension, centre influence, atari, shape balance), each labelled with the
  move of highest score under its tactical / shape heuristic, value target =
  stone balance + score / 14; 96 training samples, evaluation on samples
  8..39.  (Task constants are the reference's: train_betago_agent.py:113-251.)
* ``task="tactical"``: this project's own generator (seeded stone scatter plus
  hand-built motifs) and priority labeller (capture, rescue, atari, connect,
  3-3/4-4 framework, centre).
"""

from __future__ import annotations

import json
import sys
from dataclasses import dataclass
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import _common  # noqa: E402,F401

from underhfs import functional as F  # noqa: E402
from underhfs.nn import Linear, ReLU, Sequential  # noqa: E402
from underhfs.optim import AdamW  # noqa: E402
from underhfs.serialization import save_checkpoint  # noqa: E402
from underhfs.tensor import tensor  # noqa: E402

N = 9
POINTS = N * N
PASS = POINTS
FEATURES = 4 * POINTS
HERE = Path(__file__).resolve().parent


@dataclass(frozen=True)
class Sample:
    features: list[float]
    policy: int
    value: float
    strategy: str
    board: tuple[int, ...]


class BetaGoAgent:
    def __init__(self) -> None:
        self.trunk = Sequential(Linear(FEATURES, 32), ReLU(), Linear(32, 16), ReLU())
        self.policy_head = Linear(16, POINTS + 1)
        self.value_head = Linear(16, 1)

    def __call__(self, x):
        h = self.trunk(x)
        return self.policy_head(h), self.value_head(h)

    def parameters(self):
        for m in (self.trunk, self.policy_head, self.value_head):
            yield from m.parameters()

    def state_dict(self) -> dict:
        out = {}
        for prefix, m in (("trunk", self.trunk), ("policy", self.policy_head), ("value", self.value_head)):
            out.update({f"{prefix}.{k}": v for k, v in m.state_dict().items()})
        return out


# ------------------------------------------------------------------ rules
def adjacent(p: int) -> list[int]:
    r, c = divmod(p, N)
    return [q for q, ok in ((p - N, r > 0), (p + N, r < N - 1), (p - 1, c > 0), (p + 1, c < N - 1)) if ok]


def chain(board, p: int) -> tuple[frozenset[int], frozenset[int]]:
    """Stones connected to p and their liberties (flood fill)."""
    colour, seen, libs, todo = board[p], {p}, set(), [p]
    while todo:
        for q in adjacent(todo.pop()):
            if board[q] == 0:
                libs.add(q)
            elif board[q] == colour and q not in seen:
                seen.add(q)
                todo.append(q)
    return frozenset(seen), frozenset(libs)


def play(board, p: int, colour: int) -> tuple[int, ...] | None:
    """Board after colour plays p with captures, or None if illegal (occupied / suicide)."""
    if board[p] != 0:
        return None
    b = list(board)
    b[p] = colour
    for q in adjacent(p):
        if b[q] == -colour:
            stones, libs = chain(b, q)
            if not libs:
                for s in stones:
                    b[s] = 0
    return tuple(b) if chain(b, p)[1] else None


def legal_moves(board, colour: int) -> list[int]:
    return [p for p in range(POINTS) if play(board, p, colour) is not None] or [PASS]


# -------------------------------------------------------------- labeller
PRIORITY = ("capture", "rescue", "atari", "connect", "framework", "centre", "shape")
WEIGHT = {"capture": 12.0, "rescue": 10.0, "atari": 7.0, "connect": 5.0, "framework": 4.0, "centre": 3.0,
          "shape": 1.0, "pass": -1.0}
STAR_POINTS = {2 * N + 2, 2 * N + 6, 6 * N + 2, 6 * N + 6}


def classify(board, colour: int, move: int) -> str:
    if move == PASS:
        return "pass"
    after = play(board, move, colour)
    captured = after is not None and sum(1 for a, b in zip(board, after) if a == -colour and b == 0) > 0
    if captured:
        return "capture"
    for q in adjacent(move):
        if board[q] == colour and len(chain(board, q)[1]) == 1:
            return "rescue"
    for q in adjacent(move):
        if board[q] == -colour and len(chain(board, q)[1]) == 2 and move in chain(board, q)[1]:
            return "atari"
    if sum(1 for q in adjacent(move) if board[q] == colour) >= 2:
        return "connect"
    if move in STAR_POINTS:
        return "framework"
    r, c = divmod(move, N)
    if 3 <= r <= 5 and 3 <= c <= 5:
        return "centre"
    return "shape"


def best_move(board, colour: int) -> tuple[int, str]:
    ranked = sorted(((PRIORITY.index(classify(board, colour, m)) if m != PASS else len(PRIORITY), m)
                     for m in legal_moves(board, colour)))
    move = ranked[0][1]
    return move, classify(board, colour, move)


# ------------------------------------------------------------ positions
def scatter_position(seed: int) -> tuple[tuple[int, ...], int]:
    b = [0] * POINTS
    x = seed * 2654435761 % 2**32
    colour = 1
    for _ in range(8 + seed % 20):
        x = (1103515245 * x + 12345) % 2**31
        p = x % POINTS
        if b[p] == 0 and play(tuple(b), p, colour) is not None:
            b[p] = colour
            colour = -colour
    return tuple(b), 1 if seed % 2 == 0 else -1


def motif_position(seed: int) -> tuple[tuple[int, ...], int]:
    """Small hand-built tactical shapes around a random anchor."""
    b = [0] * POINTS
    r, c = 2 + seed % 5, 2 + (seed // 5) % 5
    a = r * N + c
    kind = seed % 4
    if kind == 0:  # opponent stone in atari next to the anchor
        b[a + 1] = -1
        for q in adjacent(a + 1):
            if q != a:
                b[q] = 1
    elif kind == 1:  # own stone in atari
        b[a] = 1
        for q in adjacent(a)[1:]:
            b[q] = -1
    elif kind == 2:  # two own stones to connect through the anchor
        b[a - 1], b[a + 1] = 1, 1
    else:  # opponent chain with two liberties
        b[a], b[a + 1] = -1, -1
        for q in set(adjacent(a) + adjacent(a + 1)) - {a, a + 1}:
            if q not in (a - 1, a + N):
                b[q] = 1
    return tuple(b), 1


def encode(board, colour: int) -> list[float]:
    legal = set(legal_moves(board, colour))
    return ([float(v == colour) for v in board] + [float(v == -colour) for v in board]
            + [float(p in legal) for p in range(POINTS)] + [float(colour)] * POINTS)


def generate_samples(count: int, offset: int = 0) -> list[Sample]:
    out = []
    for i in range(offset, offset + count):
        board, colour = motif_position(i) if i % 2 else scatter_position(i)
        move, tag = best_move(board, colour)
        value = max(-1.0, min(1.0, sum(board) * colour / POINTS + WEIGHT[tag] / 14.0))
        out.append(Sample(encode(board, colour), move, value, tag, board))
    return out


# ------------------------------------------------- the reference's task
# Score of a move under the reference labeller: tactical terms from the
# neighbouring chains (first matching term names the strategy), a positional
# term, and a small contact term.
_CHAIN_TERMS = (
    # (whose chain, liberties the chain has, base score, per-stone bonus, tag)
    (-1, 1, 9.0, 1.0, "capture"),
    (-1, 2, 3.0, 0.0, "atari"),
    (+1, 1, 8.0, 0.5, "defend_atari"),
)
_FRAMEWORK_POINTS = {(2, 2), (2, 6), (6, 2), (6, 6)}


def reference_score(board, colour: int, move: int) -> tuple[float, str]:
    if move == PASS:
        return -1.0, "pass"
    tags: list[str] = []
    total = 0.0
    for q in adjacent(move):
        if board[q] == 0:
            continue
        stones, libs = chain(board, q)
        if move not in libs:
            continue
        side = 1 if board[q] == colour else -1
        for owner, nlib, base, per_stone, tag in _CHAIN_TERMS:
            if owner == side and len(libs) == nlib:
                total += base + per_stone * len(stones)
                tags.append(tag)
                break
        else:
            if side == 1:  # own chain with two or more liberties: a connection
                total += 1.8
                tags.append("connect")
    r, c = divmod(move, N)
    edge = min(r, c, N - 1 - r, N - 1 - c)
    if (r, c) in _FRAMEWORK_POINTS:
        total += 2.4
        tags.append("corner_framework")
    elif edge == 2:
        total += 1.2
        tags.append("side_extension")
    elif 3 <= r <= 5 and 3 <= c <= 5:
        total += 1.0
        tags.append("center_influence")
    own = sum(board[q] == colour for q in adjacent(move))
    other = sum(board[q] == -colour for q in adjacent(move))
    total += 0.45 * own + 0.25 * other
    return total, (tags[0] if tags else "shape_balance")


def reference_scatter(seed: int) -> tuple[tuple[int, ...], int]:
    """Alternating stones placed by the reference's deterministic walk."""
    b = [0] * POINTS
    colour, cursor, stride = 1, (seed * 17 + 11) % POINTS, 7 + seed % 5
    for step in range(10 + seed % 18):
        for attempt in range(POINTS):
            p = (cursor + attempt * stride + step * 13) % POINTS
            if b[p] == 0:
                b[p] = colour
                break
        colour = -colour
        cursor = (cursor * 19 + 23) % POINTS
    return tuple(b), (1 if seed % 2 == 0 else -1)


# The eight strategy motifs: (move, own stones, opponent stones, tag, score),
# black to play.
_MOTIFS = (
    (40, (49,), (31, 39), "capture", 12.0),
    (40, (39, 49), (31, 41), "defend_atari", 11.0),
    (40, (39, 41), (31,), "connect", 8.0),
    (20, (19,), (11,), "corner_framework", 7.0),
    (22, (21,), (13,), "side_extension", 6.5),
    (40, (30, 50), (32, 48), "center_influence", 6.0),
    (31, (39, 49), (40,), "atari", 7.5),
    (58, (57, 67), (49,), "shape_balance", 5.5),
)


def reference_samples(count: int) -> list[Sample]:
    out = []
    for seed in range(count):
        motif = _MOTIFS[seed % 8] if seed % 8 < len(_MOTIFS) else None
        if motif is not None:
            move, own, opp, tag, score = motif
            b = [0] * POINTS
            for q in own:
                b[q] = 1
            for q in opp:
                b[q] = -1
            board, colour = tuple(b), 1
        else:
            board, colour = reference_scatter(seed)
            ranked = sorted(((reference_score(board, colour, m), m) for m in legal_moves(board, colour)),
                            key=lambda t: (t[0][0], -t[1]), reverse=True)
            (score, tag), move = ranked[0]
        value = max(-1.0, min(1.0, sum(board) * colour / POINTS + score / 14.0))
        out.append(Sample(encode(board, colour), move, value, tag, board))
    return out


def datasets(task: str) -> tuple[list[Sample], list[Sample]]:
    if task == "reference":
        return reference_samples(96), reference_samples(40)[-32:]
    if task == "tactical":
        return generate_samples(96), generate_samples(32, offset=1000)
    raise ValueError("task must be 'reference' or 'tactical'")


# ----------------------------------------------------------- training
def evaluate(model: BetaGoAgent, samples: list[Sample]) -> dict:
    logits, value = model(tensor([s.features for s in samples]))
    rows, vals = logits.tolist(), value.tolist()
    top1 = top3 = 0
    mae = 0.0
    per: dict[str, list[int]] = {}
    for s, row, v in zip(samples, rows, vals):
        order = sorted(range(len(row)), key=lambda i: -row[i])
        hit = order[0] == s.policy
        top1 += hit
        top3 += s.policy in order[:3]
        mae += abs(v[0] - s.value)
        per.setdefault(s.strategy, [0, 0])
        per[s.strategy][0] += hit
        per[s.strategy][1] += 1
    n = len(samples)
    return {"policy_top1": top1 / n, "policy_top3": top3 / n, "value_mae": mae / n,
            "strategy_accuracy": {k: w / t for k, (w, t) in sorted(per.items())}}


def train(*, steps: int = 60, batch_size: int = 8, write_artifacts: bool = True, task: str = "reference") -> dict:
    train_set, eval_set = datasets(task)
    model = BetaGoAgent()
    opt = AdamW(model.parameters(), lr=0.015, weight_decay=1e-4)
    history = []
    for step in range(steps):
        cur = [train_set[(step * batch_size + i) % len(train_set)] for i in range(batch_size)]
        logits, value = model(tensor([s.features for s in cur]))
        loss = F.cross_entropy(logits, tensor([s.policy for s in cur])) + \
            F.mse_loss(value, tensor([[s.value] for s in cur])) * 0.35
        opt.zero_grad()
        loss.backward()
        opt.step()
        if step % 10 == 0 or step == steps - 1:
            history.append({**evaluate(model, eval_set), "step": step, "loss": loss.item()})
    final = evaluate(model, eval_set)
    payload = {"task": task, "board_size": N, "train_samples": len(train_set), "eval_samples": len(eval_set),
               "steps": steps,
               "batch_size": batch_size, "final_metrics": final, "history": history,
               "strategies": sorted({s.strategy for s in train_set})}
    if write_artifacts:
        art = HERE / "artifacts"
        art.mkdir(exist_ok=True)
        state_path = art / "betago_agent_state.json"
        save_checkpoint(state_path, state=model.state_dict(),
                        metadata={"board_size": N, "features": FEATURES, "moves": POINTS + 1,
                                  "training": f"{task} strategy supervision"})
        payload["artifact"] = str(state_path.relative_to(HERE.parents[1]))
        (art / "metrics.json").write_text(json.dumps(payload, indent=2), encoding="utf-8")
    return payload


def run_smoke(*, steps: int = 5, task: str = "reference") -> dict:
    return train(steps=steps, write_artifacts=False, task=task)


if __name__ == "__main__":
    print(json.dumps(train(task=sys.argv[1] if len(sys.argv) > 1 else "reference"), indent=2))
