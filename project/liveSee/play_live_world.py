"""liveSee play server: HTTP page + JSON API over a trained LiveWorldModel.

GET /            browser page (canvas view driven by /api/state, /api/move)
GET /api/state   current chunk as JSON
GET /api/move?dir=w|a|s|d|q|e
GET /api/frame   the same view rendered headless into an RGBA device buffer by
                 the CUDA isometric rasteriser (raster.py), returned as PPM
"""

from __future__ import annotations

import json
import sys
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path
from urllib.parse import parse_qs, urlparse

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE))
import _common  # noqa: E402,F401

from underhfs.functional import cross_entropy  # noqa: E402
from underhfs.optim import SGD  # noqa: E402
from underhfs.tensor import tensor  # noqa: E402

from live_world import LiveWorldModel, move, render_chunk, spawn_player, training_samples  # noqa: E402

PAGE = """<!doctype html><html><head><meta charset="utf-8"><title>liveSee</title>
<style>body{margin:0;background:#000;color:#eee;font:13px monospace}canvas{display:block;margin:auto}
#info{position:fixed;top:8px;left:8px}</style></head><body><div id="info"></div>
<canvas id="c" width="960" height="540"></canvas><script>
const cv=document.getElementById('c'),g=cv.getContext('2d');let st=null;
function project(x,y,z,p){const dx=x-p.x,dz=z-p.z,c=Math.cos(-p.yaw),s=Math.sin(-p.yaw);
 const u=dx*c-dz*s,v=dx*s+dz*c,k=26;return[cv.width/2+(u-v)*k,cv.height*0.58+(u+v)*k*0.42-y*k];}
function tint(h,d){const n=parseInt(h.slice(1),16),f=v=>Math.max(0,Math.min(255,v+d));
 return `rgb(${f(n>>16)},${f((n>>8)&255)},${f(n&255)})`;}
function face(pts,col){g.beginPath();g.moveTo(...pts[0]);for(const q of pts.slice(1))g.lineTo(...q);g.closePath();
 g.fillStyle=col;g.fill();}
function render(){if(!st)return;const p=st.player,sky=g.createLinearGradient(0,0,0,cv.height);
 sky.addColorStop(0,'#78c7ff');sky.addColorStop(0.52,'#d8f6ff');sky.addColorStop(0.52,'#222');g.fillStyle=sky;
 g.fillRect(0,0,cv.width,cv.height);
 for(const b of [...st.blocks].sort((a,c)=>(a.x+a.y+a.z)-(c.x+c.y+c.z))){
  const P=(dx,dy,dz)=>project(b.x+dx,b.y+dy,b.z+dz,p);
  face([P(0,1,0),P(1,1,0),P(1,1,1),P(0,1,1)],b.color);face([P(0,1,1),P(1,1,1),P(1,0,1),P(0,0,1)],tint(b.color,-32));
  face([P(1,1,0),P(1,1,1),P(1,0,1),P(1,0,0)],tint(b.color,-52));}
 document.getElementById('info').textContent=`${st.prompt} x=${p.x.toFixed(1)} z=${p.z.toFixed(1)} yaw=${p.yaw.toFixed(2)}`;}
async function go(d){st=await (await fetch(d?'/api/move?dir='+d:'/api/state')).json();render();}
addEventListener('keydown',e=>{const k={arrowleft:'q',arrowright:'e'}[e.key.toLowerCase()]||e.key.toLowerCase();
 if('wasdqe'.includes(k)&&k.length==1)go(k);});go();
</script></body></html>"""


class LiveWorldSession:
    def __init__(self, prompt: str = "glowing water ruins", *, steps: int = 10) -> None:
        self.prompt = prompt
        self.player = spawn_player(prompt)
        self.model = LiveWorldModel()
        feats, labels = training_samples(prompt)
        x, y = tensor(feats), tensor(labels)
        opt = SGD(self.model.parameters(), lr=0.05)
        for _ in range(steps):
            opt.zero_grad()
            cross_entropy(self.model(x), y).backward()
            opt.step()

    def state(self) -> dict:
        return render_chunk(self.model, self.prompt, self.player, radius=8)

    def move(self, direction: str) -> dict:
        self.player = move(self.player, direction, self.prompt)
        return self.state()

    def frame(self, width: int = 960, height: int = 540):
        from raster import render_frame

        return render_frame(self.state(), width, height)


def make_handler(session: LiveWorldSession):
    class Handler(BaseHTTPRequestHandler):
        def log_message(self, *_a) -> None:
            return

        def _send(self, body: bytes, ctype: str) -> None:
            self.send_response(200)
            self.send_header("Content-Type", ctype)
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

        def do_GET(self) -> None:
            url = urlparse(self.path)
            if url.path == "/":
                return self._send(PAGE.encode("utf-8"), "text/html; charset=utf-8")
            if url.path == "/api/state":
                return self._send(json.dumps(session.state()).encode(), "application/json")
            if url.path == "/api/move":
                d = parse_qs(url.query).get("dir", [""])[0]
                return self._send(json.dumps(session.move(d)).encode(), "application/json")
            if url.path == "/api/frame":
                from raster import to_ppm

                return self._send(to_ppm(session.frame()), "image/x-portable-pixmap")
            self.send_error(404)

    return Handler


def create_server(host: str = "127.0.0.1", port: int = 8766, prompt: str = "glowing water ruins"):
    return ThreadingHTTPServer((host, port), make_handler(LiveWorldSession(prompt)))


def main() -> int:
    server = create_server()
    print("liveSee voxel world at http://127.0.0.1:8766 (WASD move, Q/E turn)")
    try:
        server.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        server.server_close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
