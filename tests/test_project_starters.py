"""The example projects run end to end on the framework."""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _load(rel: str):
    path = ROOT / rel
    sys.path.insert(0, str(path.parent))
    spec = importlib.util.spec_from_file_location(path.stem, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[path.stem] = mod  # dataclasses resolve their module by name
    spec.loader.exec_module(mod)
    return mod


def test_text2pixel():
    r = _load("project/text2image_text2pixel/train_text2pixel.py").run_smoke(steps=2)
    assert r["project"] == "text2image_text2pixel" and r["pixel_shape"] == [1, 4, 4]
    assert len(r["generated_pixels"]) == 4


def test_text2world():
    r = _load("project/text2world/train_text2world.py").run_smoke(steps=2)
    assert r["schema"] == ["agent_x", "agent_y", "goal_x", "goal_y", "resource", "hazard"]
    assert len(r["world_vector"]) == 6


def test_livesee_smoke():
    r = _load("project/liveSee/train_live_world.py").run_smoke(steps=2)
    assert r["project"] == "liveSee" and r["mode"] == "minecraft_like_voxel_world"
    assert r["task"] == "minecraft_like_ai_live_world_generation_and_play"
    assert r["controls"] == "WASD + Q/E or arrow keys"
    assert "@" in r["ascii_view"] and r["block_count"] > 0


def test_livesee_session_moves():
    mod = _load("project/liveSee/play_live_world.py")
    s = mod.LiveWorldSession(steps=1)
    before, after = s.state(), s.move("d")
    turned = s.move("e")
    assert before["mode"] == "minecraft_like_voxel_world"
    assert before["player"]["x"] == 0.0 and after["player"]["x"] == 1.0 and "z" in after["player"]
    assert turned["player"]["yaw"] > after["player"]["yaw"]
    assert len(after["blocks"]) > 0


def test_livesee_cpu_raster_frame():
    raster = _load("project/liveSee/raster.py")
    mod = _load("project/liveSee/play_live_world.py")
    frame = raster.render_frame_cpu(mod.LiveWorldSession(steps=1).state(), 320, 180)
    assert frame.shape == (180, 320)
    assert len(set(frame.ravel().tolist())) > 5  # background + shaded faces
    assert raster.to_ppm(frame).startswith(b"P6 320 180 255\n")


def test_progamer_policy():
    r = _load("project/progamer_rl/train_progamer_policy.py").run_smoke(steps=2)
    assert r["project"] == "progamer_rl" and len(r["policy"]) == 9 and len(r["oracle"]) == 9


def test_betago_smoke():
    mod = _load("project/BetaGo/train_betago_agent.py")
    r = mod.run_smoke(steps=3)
    assert 0.0 <= r["final_metrics"]["policy_top1"] <= 1.0
    assert r["final_metrics"]["value_mae"] >= 0.0
    board = tuple([0] * mod.POINTS)
    assert len(mod.legal_moves(board, 1)) == mod.POINTS


def test_betago_reference_task_reproduces_published_metrics():
    """The reference project's own BetaGo task, trained with this framework's
    Linear / AdamW / losses (CPU, fp64), lands on the metrics the reference
    publishes in project/BetaGo/artifacts/metrics.json: top-1 0.500, top-3
    0.875, value MAE 0.236 (0.23625455480191412), final loss 1.1061586872606768."""
    mod = _load("project/BetaGo/train_betago_agent.py")
    r = mod.train(write_artifacts=False, task="reference")
    m = r["final_metrics"]
    assert m["policy_top1"] == 0.5 and m["policy_top3"] == 0.875
    assert abs(m["value_mae"] - 0.23625455480191412) < 1e-9
    assert abs(r["history"][-1]["loss"] - 1.1061586872606768) < 1e-9


def test_betago_tactical_task_still_trains():
    mod = _load("project/BetaGo/train_betago_agent.py")
    r = mod.run_smoke(steps=3, task="tactical")
    assert r["task"] == "tactical" and 0.0 <= r["final_metrics"]["policy_top1"] <= 1.0
