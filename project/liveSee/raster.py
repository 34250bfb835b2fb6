"""Headless rendering of a liveSee chunk: the isometric, painter's-order view
of the browser page, drawn into an RGBA8 buffer.

``quads_for(chunk, w, h)`` projects every cube to three screen quads (top,
+z face shaded -32, +x face shaded -52) in draw order (cubes stably sorted by
x+y+z).  ``render_frame`` rasterises them with the CUDA kernel of the native
core when a GPU is present; ``render_frame_cpu`` is the CPU restatement of
the same coverage rule (pixel centre inside the convex quad, edge functions
in double precision, last quad wins) used as the oracle.
"""

from __future__ import annotations

import math

import numpy as np

SCALE, HORIZON, SQUASH = 26.0, 0.58, 0.42
FACES = (  # (corner offsets (dx, dy, dz) in order, shade)
    (((0, 1, 0), (1, 1, 0), (1, 1, 1), (0, 1, 1)), 0),
    (((0, 1, 1), (1, 1, 1), (1, 0, 1), (0, 0, 1)), -32),
    (((1, 1, 0), (1, 1, 1), (1, 0, 1), (1, 0, 0)), -52),
)


def _project(x: float, y: float, z: float, p: dict, w: int, h: int) -> tuple[float, float]:
    dx, dz = x - p["x"], z - p["z"]
    c, s = math.cos(-p["yaw"]), math.sin(-p["yaw"])
    u, v = dx * c - dz * s, dx * s + dz * c
    return w / 2 + (u - v) * SCALE, h * HORIZON + (u + v) * SCALE * SQUASH - y * SCALE


def _rgba(hexcolor: str, shade: int) -> int:
    n = int(hexcolor[1:], 16)
    r, g, b = (max(0, min(255, ((n >> k) & 255) + shade)) for k in (16, 8, 0))
    return r | (g << 8) | (b << 16) | (255 << 24)


def quads_for(chunk: dict, w: int, h: int) -> tuple[np.ndarray, np.ndarray]:
    p = chunk["player"]
    cubes = sorted(chunk["blocks"], key=lambda b: b["x"] + b["y"] + b["z"])  # stable
    quads, colors = [], []
    for b in cubes:
        for corners, shade in FACES:
            pts = [_project(b["x"] + dx, b["y"] + dy, b["z"] + dz, p, w, h) for dx, dy, dz in corners]
            quads.append([c for pt in pts for c in pt])
            colors.append(_rgba(b["color"], shade))
    return np.asarray(quads, dtype=np.float32).reshape(-1, 8), np.asarray(colors, dtype=np.uint32)


def _background(w: int, h: int) -> np.ndarray:
    t = (np.arange(h, dtype=np.float32) + 0.5) / np.float32(h)
    u = t / np.float32(0.52)
    r = (0x78 + (0xD8 - 0x78) * u + 0.5).astype(np.uint32)
    g = (0xC7 + (0xF6 - 0xC7) * u + 0.5).astype(np.uint32)
    b = np.full(h, 0xFF, dtype=np.uint32)
    sky = r | (g << 8) | (b << 16) | np.uint32(0xFF << 24)
    ground = np.uint32(0x22 | (0x22 << 8) | (0x22 << 16) | (0xFF << 24))
    col = np.where(t < 0.52, sky, ground)
    return np.repeat(col[:, None], w, axis=1)


def render_frame_cpu(chunk: dict, w: int = 960, h: int = 540) -> np.ndarray:
    quads, colors = quads_for(chunk, w, h)
    order = np.zeros((h, w), dtype=np.int64)
    for q in range(len(quads)):
        pts = quads[q].reshape(4, 2).astype(np.float64)
        x0, x1 = max(0, int(math.floor(pts[:, 0].min()))), min(w - 1, int(math.ceil(pts[:, 0].max())))
        y0, y1 = max(0, int(math.floor(pts[:, 1].min()))), min(h - 1, int(math.ceil(pts[:, 1].max())))
        if x0 > x1 or y0 > y1:
            continue
        px, py = np.meshgrid(np.arange(x0, x1 + 1) + 0.5, np.arange(y0, y1 + 1) + 0.5)
        pos = np.ones_like(px, dtype=bool)
        neg = np.ones_like(px, dtype=bool)
        for e in range(4):
            (ax, ay), (bx, by) = pts[e], pts[(e + 1) % 4]
            v = (bx - ax) * (py - ay) - (by - ay) * (px - ax)
            pos &= v >= 0
            neg &= v <= 0
        cover = pos | neg
        region = order[y0 : y1 + 1, x0 : x1 + 1]
        region[cover] = np.maximum(region[cover], q + 1)
    out = _background(w, h)
    hit = order > 0
    out[hit] = colors[order[hit] - 1]
    return out


def render_frame(chunk: dict, w: int = 960, h: int = 540) -> np.ndarray:
    """GPU rasterisation when a CUDA device is present, else the CPU path."""
    try:
        import torch

        from underhfs_b200.native import status
        from underhfs_b200.ops._lib import core

        if not status().cuda_enabled:
            return render_frame_cpu(chunk, w, h)
        quads, colors = quads_for(chunk, w, h)
        q = torch.from_numpy(quads).cuda()
        c = torch.from_numpy(colors.view(np.int32)).cuda()
        order = torch.empty(h * w, dtype=torch.int32, device="cuda")
        rgba = torch.empty(h * w, dtype=torch.int32, device="cuda")
        core().raster_iso(q.data_ptr(), c.data_ptr(), len(quads), order.data_ptr(), rgba.data_ptr(), w, h,
                          torch.cuda.current_stream().cuda_stream)
        return rgba.cpu().numpy().view(np.uint32).reshape(h, w)
    except ImportError:
        return render_frame_cpu(chunk, w, h)


def to_ppm(rgba: np.ndarray) -> bytes:
    h, w = rgba.shape
    rgb = np.stack([(rgba >> s) & 255 for s in (0, 8, 16)], axis=-1).astype(np.uint8)
    return f"P6 {w} {h} 255\n".encode("ascii") + rgb.tobytes()
