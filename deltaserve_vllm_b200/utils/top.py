"""dserve-top: a live dashboard for a running server (stdlib only).

    python -m deltaserve_vllm_b200.utils.top --server http://127.0.0.1:8000 --port 8090
    python -m deltaserve_vllm_b200.utils.top --replay run.json --port 8090

It polls the server's ``/telemetry/data`` (step stream + per-window series),
``/system_metrics`` and ``/finetuning_status``, keeps a history (capped by
``--history-hours``), and serves one HTML page that redraws every poll:
throughput of inference and finetuning tokens, TTFT / TBT percentiles and SLO
attainment, the latest steps (composition, predicted vs measured GPU time),
and the finetuning state. ``/api/export`` downloads the history as JSON;
``--replay`` serves such a file without a server. On start it asks the server
to start telemetry (``POST /telemetry/start``) unless ``--no-start``.
Reference: ``deltaserve-plugin/deltaserve/top.py:484-550`` (same roles:
poll, record, export, replay).
"""

from __future__ import annotations

import argparse
import json
import threading
import time
import urllib.request
from collections import deque
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

PAGE = """<!doctype html><html><head><meta charset="utf-8"><title>dserve-top</title>
<style>body{font:13px monospace;background:#111;color:#ddd;margin:16px}
h2{margin:6px 0;color:#8cf}table{border-collapse:collapse}td,th{padding:2px 8px;border-bottom:1px solid #333}
.k{color:#999}.ok{color:#6d6}.bad{color:#f66}svg{background:#1a1a1a}</style></head><body>
<h2>dserve-top <span id=src class=k></span></h2>
<div id=sum></div><svg id=tp width=900 height=160></svg>
<h2>finetuning</h2><div id=ft></div><h2>steps</h2><table id=steps></table>
<script>
function line(svg,pts,color,ymax){let w=svg.width.baseVal.value,h=svg.height.baseVal.value;
 if(pts.length<2)return '';let x0=pts[0][0],x1=pts[pts.length-1][0]||x0+1;
 let d=pts.map((p,i)=>(i?'L':'M')+((p[0]-x0)/(x1-x0+1e-9)*w).toFixed(1)+','+(h-p[1]/(ymax||1)*h*0.95).toFixed(1)).join('');
 return `<path d="${d}" stroke="${color}" fill="none"/>`}
async function tick(){let r=await fetch('/api/data');let d=await r.json();
 document.getElementById('src').textContent=d.source;
 let s=(d.metrics||{}).current||{};let fmt=v=>v==null?'-':(typeof v=='number'?v.toFixed(3):v);
 document.getElementById('sum').innerHTML=`<table><tr><th>inf tok/s</th><th>ft tok/s</th><th>TTFT p50/p99 (s)</th><th>TBT p50/p99 (s)</th><th>SLO attainment</th><th>requests</th></tr>
 <tr><td>${fmt(s.inf_tok_s)}</td><td>${fmt(s.ft_tok_s)}</td><td>${fmt(s.ttft_p50_s)} / ${fmt(s.ttft_p99_s)}</td><td>${fmt(s.tbt_p50_s)} / ${fmt(s.tbt_p99_s)}</td>
 <td class="${(s.slo_attainment??1)>=0.99?'ok':'bad'}">${fmt(s.slo_attainment)}</td><td>${fmt(s.requests)}</td></tr></table>`;
 let ser=d.series||[];let m=Math.max(1,...ser.map(p=>Math.max(p[1],p[2])));
 let svg=document.getElementById('tp');svg.innerHTML=line(svg,ser.map(p=>[p[0],p[1]]),'#6cf',m)+line(svg,ser.map(p=>[p[0],p[2]]),'#fc6',m);
 document.getElementById('ft').innerHTML='<pre>'+JSON.stringify(d.finetuning||{},null,1).slice(0,1500)+'</pre>';
 let rows=(d.steps||[]).slice(-30).reverse().map(x=>`<tr><td>${x.seq}</td><td>${x.kind}</td><td>${x.t_in}</td><td>${x.t_ft}</td><td>${x.b_d}</td><td>${x.gpu_ms}</td><td>${x.pred_ms??'-'}</td><td>${x.n??1}</td><td>${x.bwd?'bwd':''}</td></tr>`).join('');
 document.getElementById('steps').innerHTML='<tr><th>seq</th><th>kind</th><th>t_in</th><th>t_ft</th><th>b_d</th><th>gpu ms</th><th>pred ms</th><th>n</th><th></th></tr>'+rows;}
setInterval(tick,1000);tick();
</script></body></html>"""


class Recorder:
    def __init__(self, server: str | None, history_hours: float = 12.0, poll_s: float = 1.0):
        self.server = server.rstrip("/") if server else None
        self.poll_s = poll_s
        self.steps: deque = deque(maxlen=20000)
        self.series: deque = deque(maxlen=int(history_hours * 3600))
        self.metrics: dict = {}
        self.finetuning: dict = {}
        self.last_seq = 0
        self.source = server or "replay"
        self._lock = threading.Lock()
        self._stop = threading.Event()

    def _get(self, path: str, body: dict | None = None):
        req = urllib.request.Request(self.server + path, method="POST" if body is not None else "GET",
                                     data=json.dumps(body).encode() if body is not None else None,
                                     headers={"content-type": "application/json"})
        with urllib.request.urlopen(req, timeout=5) as r:
            return json.loads(r.read().decode())

    def start_telemetry(self) -> None:
        try:
            self._get("/telemetry/start", {})
        except Exception:
            pass

    def poll_once(self) -> None:
        data = self._get(f"/telemetry/data?steps_since={self.last_seq}")
        met = self._get("/system_metrics")
        ft = self._get("/finetuning_status")
        with self._lock:
            for s in data.get("steps", []):
                self.steps.append(s)
                self.last_seq = max(self.last_seq, int(s.get("seq", 0)))
            cur = met.get("current") or {}
            self.series.append((time.time(), float(cur.get("inf_tok_s") or 0), float(cur.get("ft_tok_s") or 0)))
            self.metrics, self.finetuning = met, ft

    def run(self) -> None:
        while not self._stop.is_set():
            try:
                self.poll_once()
            except Exception:
                pass
            self._stop.wait(self.poll_s)

    def snapshot(self) -> dict:
        with self._lock:
            return {"source": self.source, "steps": list(self.steps)[-200:], "series": list(self.series),
                    "metrics": self.metrics, "finetuning": self.finetuning}

    def export(self) -> dict:
        with self._lock:
            return {"source": self.source, "steps": list(self.steps), "series": list(self.series),
                    "metrics": self.metrics, "finetuning": self.finetuning}

    def load(self, path: str) -> None:
        with open(path) as f:
            d = json.load(f)
        self.steps.extend(d.get("steps", []))
        self.series.extend(tuple(x) for x in d.get("series", []))
        self.metrics, self.finetuning = d.get("metrics", {}), d.get("finetuning", {})
        self.source = f"replay of {path}"


def make_handler(rec: Recorder):
    class H(BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def _send(self, code: int, body: bytes, ctype: str, extra: dict | None = None):
            self.send_response(code)
            self.send_header("content-type", ctype)
            for k, v in (extra or {}).items():
                self.send_header(k, v)
            self.end_headers()
            self.wfile.write(body)

        def do_GET(self):
            if self.path == "/":
                self._send(200, PAGE.encode(), "text/html")
            elif self.path == "/api/data":
                self._send(200, json.dumps(rec.snapshot()).encode(), "application/json")
            elif self.path == "/api/export":
                self._send(200, json.dumps(rec.export()).encode(), "application/json",
                           {"content-disposition": "attachment; filename=dserve-top.json"})
            else:
                self._send(404, b"not found", "text/plain")
    return H


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--server", default="http://127.0.0.1:8000")
    ap.add_argument("--port", type=int, default=8090)
    ap.add_argument("--bind", default="127.0.0.1")
    ap.add_argument("--poll", type=float, default=1.0, help="seconds between polls")
    ap.add_argument("--history-hours", type=float, default=12.0)
    ap.add_argument("--replay", default=None, help="serve an exported JSON instead of polling")
    ap.add_argument("--no-start", action="store_true", help="do not POST /telemetry/start")
    args = ap.parse_args(argv)
    rec = Recorder(None if args.replay else args.server, args.history_hours, args.poll)
    if args.replay:
        rec.load(args.replay)
    else:
        if not args.no_start:
            rec.start_telemetry()
        threading.Thread(target=rec.run, daemon=True).start()
    srv = ThreadingHTTPServer((args.bind, args.port), make_handler(rec))
    print(f"dserve-top on http://{args.bind}:{args.port} ({rec.source})", flush=True)
    try:
        srv.serve_forever()
    except KeyboardInterrupt:
        pass


if __name__ == "__main__":
    main()
