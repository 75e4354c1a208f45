"""Model hub downloads with integrity checks (Hugging Face hub API layout).

``pull(repo_id)`` lists a repository revision's files (``GET {endpoint}/api/models/{repo}/revision/
{rev}?blobs=true``), picks the serving files (config / tokenizer / safetensors / GGUF by default, or
``allow`` glob patterns), and downloads each one from ``{endpoint}/{repo}/resolve/{rev}/{file}``
into ``$GOLLEK_HOME/models/{repo}`` (or ``dest``):

* resumable: a ``.part`` file continues with an HTTP ``Range`` request after an interruption;
* verified: LFS files against the listing's sha256, other files against their listed size;
  a mismatch deletes the file and raises;
* recorded: ``gollek-manifest.json`` keeps each file's size and sha256 so a second ``pull``
  skips files that are already complete and ``verify(dir)`` can re-check a local copy.

``HF_ENDPOINT`` overrides the endpoint and ``HF_TOKEN`` (or ``token``) is sent as a bearer token
for gated repositories. Reference: repository/gollek-model-repo-hf/…/repo/hf/HuggingFaceClient.java
(:59-61 listing with siblings, :141 resolve URL, :322 bearer token) and HuggingFaceDownloader.java.
"""
from __future__ import annotations

import fnmatch
import hashlib
import json
import os
from typing import Callable, Dict, List, Optional

DEFAULT_ALLOW = ["*.json", "*.safetensors", "*.gguf", "tokenizer.model", "*.txt", "*.jinja"]
MANIFEST = "gollek-manifest.json"


class HubError(RuntimeError):
    pass


def _home() -> str:
    return os.environ.get("GOLLEK_HOME", os.path.expanduser("~/.gollek"))


def _sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 22), b""):
            h.update(chunk)
    return h.hexdigest()


class HubClient:
    def __init__(self, endpoint: Optional[str] = None, token: Optional[str] = None, timeout_s: float = 60.0):
        import requests
        self.endpoint = (endpoint or os.environ.get("HF_ENDPOINT") or "https://huggingface.co").rstrip("/")
        self.token = token or os.environ.get("HF_TOKEN")
        self.timeout_s = timeout_s
        self.http = requests.Session()

    def _headers(self, extra: Optional[dict] = None) -> dict:
        h = {"User-Agent": "gollek-b200"}
        if self.token:
            h["Authorization"] = f"Bearer {self.token}"
        h.update(extra or {})
        return h

    def list_files(self, repo_id: str, revision: str = "main") -> List[dict]:
        """[{"name", "size", "sha256" (LFS files) or None}] of a repository revision."""
        url = f"{self.endpoint}/api/models/{repo_id}/revision/{revision}"
        r = self.http.get(url, params={"blobs": "true"}, headers=self._headers(), timeout=self.timeout_s)
        if r.status_code == 401 or r.status_code == 403:
            raise HubError(f"{repo_id}: access denied (gated repository? set HF_TOKEN)")
        if r.status_code == 404:
            raise HubError(f"{repo_id}@{revision}: not found")
        r.raise_for_status()
        out = []
        for s in r.json().get("siblings", []):
            lfs = s.get("lfs") or {}
            out.append({"name": s["rfilename"], "size": lfs.get("size", s.get("size")),
                        "sha256": lfs.get("sha256")})
        return out

    def download(self, repo_id: str, f: dict, dest_dir: str, revision: str = "main",
                 progress: Optional[Callable[[str, int, Optional[int]], None]] = None) -> Dict[str, object]:
        """One file, resumed from ``<name>.part`` when present; verified; returns its manifest entry."""
        name = f["name"]
        path = os.path.join(dest_dir, name)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        part = path + ".part"
        have = os.path.getsize(part) if os.path.exists(part) else 0
        url = f"{self.endpoint}/{repo_id}/resolve/{revision}/{name}"
        hdr = {"Range": f"bytes={have}-"} if have else {}
        with self.http.get(url, headers=self._headers(hdr), stream=True, timeout=self.timeout_s) as r:
            if r.status_code == 416:  # the .part already holds the whole file
                pass
            else:
                if r.status_code not in (200, 206):
                    raise HubError(f"{name}: HTTP {r.status_code}")
                mode = "ab" if (have and r.status_code == 206) else "wb"
                done = have if mode == "ab" else 0
                with open(part, mode) as out:
                    for chunk in r.iter_content(1 << 16):
                        out.write(chunk)
                        done += len(chunk)
                        if progress is not None:
                            progress(name, done, f.get("size"))
        size = os.path.getsize(part)
        if f.get("size") is not None and size != int(f["size"]):
            os.remove(part)
            raise HubError(f"{name}: size {size} != listed {f['size']}")
        digest = _sha256(part)
        if f.get("sha256") and digest != f["sha256"]:
            os.remove(part)
            raise HubError(f"{name}: sha256 mismatch (got {digest[:12]}…, listed {f['sha256'][:12]}…)")
        os.replace(part, path)
        return {"size": size, "sha256": digest, "verified": "sha256" if f.get("sha256") else "size"}


def _selected(files: List[dict], allow: Optional[List[str]]) -> List[dict]:
    pats = allow or DEFAULT_ALLOW
    return [f for f in files if any(fnmatch.fnmatch(os.path.basename(f["name"]), p) or fnmatch.fnmatch(f["name"], p)
                                    for p in pats)]


def pull(repo_id: str, revision: str = "main", dest: Optional[str] = None, allow: Optional[List[str]] = None,
         endpoint: Optional[str] = None, token: Optional[str] = None,
         progress: Optional[Callable[[str, int, Optional[int]], None]] = None) -> str:
    """Download (or complete) a repository revision; returns the local directory."""
    client = HubClient(endpoint, token)
    dest = dest or os.path.join(_home(), "models", repo_id)
    os.makedirs(dest, exist_ok=True)
    mpath = os.path.join(dest, MANIFEST)
    manifest = {"repo_id": repo_id, "revision": revision, "files": {}}
    if os.path.exists(mpath):
        with open(mpath) as fh:
            old = json.load(fh)
        if old.get("repo_id") == repo_id and old.get("revision") == revision:
            manifest = old
    for f in _selected(client.list_files(repo_id, revision), allow):
        entry = manifest["files"].get(f["name"])
        path = os.path.join(dest, f["name"])
        if (entry and os.path.exists(path) and os.path.getsize(path) == entry["size"]
                and (not f.get("sha256") or entry["sha256"] == f["sha256"])):
            continue  # complete from an earlier pull
        manifest["files"][f["name"]] = client.download(repo_id, f, dest, revision, progress)
        with open(mpath, "w") as fh:
            json.dump(manifest, fh, indent=1)
    with open(mpath, "w") as fh:
        json.dump(manifest, fh, indent=1)
    return dest


def verify(directory: str) -> Dict[str, str]:
    """Re-check a pulled directory against its manifest: {file: "ok" | "missing" | "corrupt"}."""
    with open(os.path.join(directory, MANIFEST)) as fh:
        manifest = json.load(fh)
    out = {}
    for name, e in manifest["files"].items():
        p = os.path.join(directory, name)
        if not os.path.exists(p):
            out[name] = "missing"
        elif os.path.getsize(p) != e["size"] or _sha256(p) != e["sha256"]:
            out[name] = "corrupt"
        else:
            out[name] = "ok"
    return out
