"""OpenAI audio endpoints: POST /v1/audio/speech over a SpeechT5 + HiFi-GAN model (text to WAV), and
over a Whisper model POST /v1/audio/transcriptions and /v1/audio/translations (multipart ``file``, ``model``, ``language``, ``prompt``, ``response_format``
json | text | verbose_json | srt | vtt, ``temperature``).

Requests that arrive together are batched: one worker thread takes every pending upload with the
same (task, language, temperature, timestamps) and runs them as one ``WhisperASR.transcribe`` call,
so their 30 s windows share the encoder GEMMs and the decode steps.

Reference: runner/safetensor/gollek-safetensor-api/…/api/AudioResource.java (:54 transcriptions,
:98 translations; form fields file / model / language / temperature / response_format / prompt).
"""
from __future__ import annotations

import asyncio
import queue
import threading
from typing import Any, Dict, List, Optional

from fastapi import FastAPI, File, Form, HTTPException, UploadFile
from fastapi.responses import JSONResponse, PlainTextResponse, Response

FORMATS = ("json", "text", "verbose_json", "srt", "vtt")


def _clock(t: float, sep: str) -> str:
    ms = int(round(t * 1000))
    h, ms = divmod(ms, 3600_000)
    m, ms = divmod(ms, 60_000)
    s, ms = divmod(ms, 1000)
    return f"{h:02d}:{m:02d}:{s:02d}{sep}{ms:03d}"


def subtitles(segments: List[dict], kind: str) -> str:
    """SubRip (``srt``) or WebVTT (``vtt``) text of timed segments."""
    sep = "," if kind == "srt" else "."
    out = [] if kind == "srt" else ["WEBVTT", ""]
    for i, s in enumerate(segments, 1):
        if kind == "srt":
            out.append(str(i))
        out += [f"{_clock(s['start'], sep)} --> {_clock(s['end'], sep)}", s["text"], ""]
    return "\n".join(out)


class ASRBatcher:
    """Batches concurrent transcription requests onto one worker thread."""

    def __init__(self, asr, max_batch: int = 32):
        self.asr, self.max_batch = asr, max_batch
        self.q: "queue.Queue" = queue.Queue()
        self._t = threading.Thread(target=self._loop, name="gollek-asr", daemon=True)
        self._t.start()

    async def submit(self, audio: bytes, **kw) -> dict:
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        self.q.put((audio, kw, loop, fut))
        return await fut

    def _loop(self) -> None:
        while True:
            first = self.q.get()
            if first is None:
                return
            batch = [first]
            while len(batch) < self.max_batch:
                try:
                    nxt = self.q.get_nowait()
                except queue.Empty:
                    break
                if nxt is None:
                    self.q.put(None)
                    break
                batch.append(nxt)
            groups: Dict[tuple, list] = {}
            for item in batch:
                groups.setdefault(tuple(sorted(item[1].items())), []).append(item)
            for key, items in groups.items():
                try:
                    res = self.asr.transcribe([i[0] for i in items], **dict(key))
                    for (_, _, loop, fut), r in zip(items, res):
                        loop.call_soon_threadsafe(fut.set_result, r)
                except Exception as e:  # a bad file fails its group only
                    for _, _, loop, fut in items:
                        loop.call_soon_threadsafe(fut.set_exception, e)

    def close(self) -> None:
        self.q.put(None)


def register_audio_routes(app: FastAPI, asr, tts=None) -> Optional[ASRBatcher]:
    """Mount the audio endpoints (501 when the model they need is not loaded). ``tts``: a
    ``SpeechSynth`` behind POST /v1/audio/speech (JSON ``input``, ``voice``, ``response_format``
    wav | pcm, ``seed``; the response is the audio bytes)."""
    batcher = ASRBatcher(asr) if asr is not None else None
    tts_lock = threading.Lock()

    @app.post("/v1/audio/speech")
    async def speech(body: Dict[str, Any]):
        if tts is None:
            raise HTTPException(501, "no text-to-speech model loaded (serve with --tts-model / --tts-vocoder)")
        text = body.get("input")
        fmt = body.get("response_format", "wav")
        if not isinstance(text, str) or not text.strip():
            raise HTTPException(400, "input must be a non-empty string")
        if fmt not in ("wav", "pcm"):
            raise HTTPException(400, "response_format must be wav or pcm")

        def run():
            with tts_lock:  # one synthesis at a time on the model's device
                return tts.wav_bytes(text, body.get("voice"), int(body.get("seed", 0)))
        try:
            data = await asyncio.get_running_loop().run_in_executor(None, run)
        except ValueError as e:
            raise HTTPException(400, str(e))
        if fmt == "pcm":  # raw 16-bit little-endian samples after the 44-byte WAVE header
            return Response(content=data[44:], media_type="audio/pcm")
        return Response(content=data, media_type="audio/wav")

    async def run(task: str, file: UploadFile, language: Optional[str], response_format: str,
                  temperature: float):
        if batcher is None:
            raise HTTPException(501, "no speech-recognition model loaded (serve with --asr-model)")
        if response_format not in FORMATS:
            raise HTTPException(400, f"response_format must be one of {', '.join(FORMATS)}")
        data = await file.read()
        timed = response_format in ("srt", "vtt")
        try:
            r = await batcher.submit(data, language=language or None, task=task, timestamps=timed,
                                     temperature=float(temperature or 0.0))
        except ValueError as e:
            raise HTTPException(400, str(e))
        if response_format == "text":
            return PlainTextResponse(r["text"])
        if timed:
            return PlainTextResponse(subtitles(r["segments"], response_format))
        if response_format == "verbose_json":
            body: Dict[str, Any] = {"task": task + ("d" if task == "translate" else ""), "language": r["language"],
                                    "duration": r["duration"], "text": r["text"],
                                    "segments": [{"id": i, **s} for i, s in enumerate(r["segments"])]}
            return JSONResponse(body)
        return JSONResponse({"text": r["text"]})

    @app.post("/v1/audio/transcriptions")
    async def transcriptions(file: UploadFile = File(...), model: Optional[str] = Form(None),
                             language: Optional[str] = Form(None), prompt: Optional[str] = Form(None),
                             response_format: str = Form("json"), temperature: float = Form(0.0)):
        return await run("transcribe", file, language, response_format, temperature)

    @app.post("/v1/audio/translations")
    async def translations(file: UploadFile = File(...), model: Optional[str] = Form(None),
                           prompt: Optional[str] = Form(None), response_format: str = Form("json"),
                           temperature: float = Form(0.0)):
        return await run("translate", file, None, response_format, temperature)

    return batcher
