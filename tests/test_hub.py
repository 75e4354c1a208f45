"""Hub downloads against a local fake hub: listing, selection, sha256 / size verification, resume
with Range after an interruption, skip on a second pull, manifest re-verification, CLI."""
import hashlib
import json
import os
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import pytest

from gollek_b200.utils import hub


def _server(files, lfs=("model.safetensors",), fail_once=None, corrupt=None):
    state = {"failed": False, "ranges": []}

    class H(BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def do_GET(self):
            if self.path.startswith("/api/models/org/tiny/revision/main"):
                sib = []
                for n, data in files.items():
                    e = {"rfilename": n, "size": len(data)}
                    if n in lfs:
                        e["lfs"] = {"sha256": hashlib.sha256(data).hexdigest(), "size": len(data)}
                    sib.append(e)
                body = json.dumps({"id": "org/tiny", "siblings": sib}).encode()
                self.send_response(200)
                self.send_header("Content-Length", str(len(body)))
                self.end_headers()
                self.wfile.write(body)
                return
            pre = "/org/tiny/resolve/main/"
            if not self.path.startswith(pre):
                self.send_response(404)
                self.end_headers()
                return
            name = self.path[len(pre):]
            data = files[name]
            if corrupt == name:
                data = data[:-1] + bytes([data[-1] ^ 1])
            start = 0
            rng = self.headers.get("Range")
            if rng:
                start = int(rng.split("=")[1].split("-")[0])
                state["ranges"].append((name, start))
            chunk = data[start:]
            self.send_response(206 if rng else 200)
            self.send_header("Content-Length", str(len(chunk)))
            self.end_headers()
            if fail_once == name and not state["failed"]:
                state["failed"] = True
                self.wfile.write(chunk[: len(chunk) // 2])  # then drop the connection
                self.wfile.flush()
                self.connection.shutdown(2)
                return
            self.wfile.write(chunk)

    srv = ThreadingHTTPServer(("127.0.0.1", 0), H)
    srv.daemon_threads = True
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv, state


FILES = {"config.json": b'{"model_type": "llama"}', "model.safetensors": os.urandom(300_000),
         "README.md": b"not a serving file", "sub/tokenizer.json": b"{}"}


def test_pull_verify_and_skip(tmp_path):
    srv, _ = _server(FILES)
    ep = f"http://127.0.0.1:{srv.server_address[1]}"
    d = hub.pull("org/tiny", dest=str(tmp_path / "m"), endpoint=ep)
    assert sorted(os.listdir(d)) == ["config.json", "gollek-manifest.json", "model.safetensors", "sub"]
    with open(os.path.join(d, "model.safetensors"), "rb") as f:
        assert f.read() == FILES["model.safetensors"]
    m = json.load(open(os.path.join(d, "gollek-manifest.json")))
    assert m["files"]["model.safetensors"]["verified"] == "sha256" and m["files"]["config.json"]["verified"] == "size"
    assert all(v == "ok" for v in hub.verify(d).values())
    mt = os.path.getmtime(os.path.join(d, "model.safetensors"))
    hub.pull("org/tiny", dest=d, endpoint=ep)  # complete files are skipped
    assert os.path.getmtime(os.path.join(d, "model.safetensors")) == mt
    with open(os.path.join(d, "config.json"), "wb") as f:
        f.write(b"tampered!")
    assert hub.verify(d)["config.json"] == "corrupt"
    srv.shutdown()


def test_checksum_mismatch_is_rejected(tmp_path):
    srv, _ = _server(FILES, corrupt="model.safetensors")
    ep = f"http://127.0.0.1:{srv.server_address[1]}"
    with pytest.raises(hub.HubError, match="sha256 mismatch"):
        hub.pull("org/tiny", dest=str(tmp_path / "m"), endpoint=ep)
    assert not os.path.exists(tmp_path / "m" / "model.safetensors")
    srv.shutdown()


def test_interrupted_download_resumes_with_range(tmp_path):
    srv, state = _server(FILES, fail_once="model.safetensors")
    ep = f"http://127.0.0.1:{srv.server_address[1]}"
    with pytest.raises(Exception):
        hub.pull("org/tiny", dest=str(tmp_path / "m"), endpoint=ep)
    assert os.path.exists(tmp_path / "m" / "model.safetensors.part")
    d = hub.pull("org/tiny", dest=str(tmp_path / "m"), endpoint=ep)
    assert state["ranges"] and state["ranges"][0][0] == "model.safetensors" and state["ranges"][0][1] > 0
    with open(os.path.join(d, "model.safetensors"), "rb") as f:
        assert f.read() == FILES["model.safetensors"]
    srv.shutdown()
