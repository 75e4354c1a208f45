"""Command-line interface: ``python -m gollek_b200 <command>``.

Commands follow the reference CLI (ui/gollek-cli/…/cli/commands/RunCommand.java:45-324 and
siblings: run, chat, batch, list, show, convert, quantize, serve, providers, stats, pull; plus
transcribe and speak for audio):

  run       one-shot generation            chat      interactive chat loop
  batch     JSONL prompts → JSONL outputs  serve     HTTP server (OpenAI + gollek routes)
  convert   safetensors → GGUF (F32/F16/Q8_0/Q4_K)
  quantize  GGUF → GGUF at another type, or safetensors → block-scaled FP8 / AWQ / AutoRound / QuIP
  show      model config and tensor table  list      presets and models under $GOLLEK_HOME
  bench     serving benchmark (bench.py)
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time


def _engine(args):
    from .config import EngineConfig
    from .engine.engine import LLMEngine
    over = dict(model=args.model)
    if getattr(args, "device", None):
        over["device"] = args.device
    if getattr(args, "max_model_len", None):
        over["max_model_len"] = args.max_model_len
    if getattr(args, "device", None) == "cpu":
        over["dtype"] = "float32"
        over["use_cuda_graphs"] = False
    cfg = EngineConfig.load(getattr(args, "config", None), **over)
    return LLMEngine(cfg)


def _params(args):
    from .engine.sequence import SamplingParams
    return SamplingParams(temperature=args.temperature, top_p=args.top_p, top_k=args.top_k,
                          max_tokens=args.max_tokens, seed=args.seed).validate()


def cmd_run(args):
    eng = _engine(args)
    t0 = time.perf_counter()
    out = eng.generate([args.prompt], _params(args))[0]
    dt = time.perf_counter() - t0
    text = out.text or (eng.tokenizer.decode(out.output_token_ids) if eng.tokenizer else str(out.output_token_ids))
    print(text)
    if args.stats:
        n = len(out.output_token_ids)
        print(f"\n[{n} tokens in {dt:.2f}s, {n / dt:.1f} tok/s, finish={out.finish_reason}]", file=sys.stderr)


def cmd_chat(args):
    eng = _engine(args)
    history = []
    print("chat (empty line or Ctrl-D to quit)")
    for line in sys.stdin:
        line = line.rstrip("\n")
        if not line:
            break
        history.append({"role": "user", "content": line})
        prompt = eng.tokenizer.apply_chat_template(history)
        out = eng.generate([prompt], _params(args))[0]
        text = out.text or eng.tokenizer.decode(out.output_token_ids)
        history.append({"role": "assistant", "content": text})
        print(text, flush=True)


def cmd_batch(args):
    eng = _engine(args)
    prompts = [json.loads(l)["prompt"] for l in open(args.input) if l.strip()]
    outs = eng.generate(prompts, _params(args))
    with open(args.output, "w") as f:
        for p, o in zip(prompts, outs):
            text = o.text or (eng.tokenizer.decode(o.output_token_ids) if eng.tokenizer else "")
            f.write(json.dumps({"prompt": p, "text": text, "tokens": o.output_token_ids,
                                "finish_reason": o.finish_reason}) + "\n")
    print(f"wrote {len(outs)} results to {args.output}")


def cmd_serve(args):
    from .server.__main__ import main as serve_main
    serve_main(sys.argv[2:])


def cmd_convert(args):
    import torch
    from .config import ModelConfig
    from .loaders import gguf as G
    from .loaders.safetensors import SafetensorsCheckpoint
    with open(os.path.join(args.src, "config.json")) as f:
        cfg = ModelConfig.from_hf(json.load(f))
    ck = SafetensorsCheckpoint(args.src)
    w = {k: ck.get(k).float() for k in ck.keys()}
    t = args.type.upper()
    t = t if t in G.MIXTURES else G.TYPE_BY_NAME[t]
    emb = G.TYPE_BY_NAME[args.embed_type.upper()] if args.embed_type else None
    G.write_llama_gguf(args.dst, cfg, w, t, embed_type=emb)
    print(f"wrote {args.dst} ({args.type})")


def cmd_quantize(args):
    from .loaders import gguf as G
    if args.src.endswith(".gguf"):
        cfg, w, f = G.load_llama_gguf(args.src)
        t = args.type.upper()
        G.write_llama_gguf(args.dst, cfg, w, t if t in G.MIXTURES else G.TYPE_BY_NAME[t])
        print(f"wrote {args.dst} ({args.type})")
    elif args.method in ("awq", "autoround", "quip", "nvfp4", "mxfp4"):
        from .quant.offline import quantize_checkpoint
        calib = None
        if args.calib_file:  # one calibration sequence of token ids per line
            with open(args.calib_file) as f:
                calib = [[int(t) for t in ln.split()] for ln in f if ln.strip()]
        r = quantize_checkpoint(args.src, args.dst, args.method, group=args.group, calib_ids=calib,
                                iters=args.iters, stages=args.stages)
        print(f"wrote {args.dst} ({r['method']}: {r['linears']} linears quantized)")
    else:
        from .quant.fp8 import quantize_checkpoint_fp8
        quantize_checkpoint_fp8(args.src, args.dst)
        print(f"wrote {args.dst} (fp8 e4m3, 128x128 block scales)")


def cmd_dequantize(args):
    """A GPTQ / AWQ / AutoRound 4-bit or QuIP checkpoint directory -> dense bf16 safetensors (plus its
    config.json without the quantization block), for tools that need plain weights."""
    import shutil

    import torch
    from .loaders.safetensors import SafetensorsCheckpoint, save_sharded
    from .quant.int4 import QUANT_METHODS, Int4Weight, checkpoint_quant_config, quantized_checkpoint_getter
    with open(os.path.join(args.src, "config.json")) as f:
        hf = json.load(f)
    qc = checkpoint_quant_config(args.src)
    if not qc or qc.get("quant_method") not in QUANT_METHODS:
        raise SystemExit(f"{args.src}: no supported quantization_config in config.json / hf_quant_config.json")
    ck = SafetensorsCheckpoint(args.src)
    get = quantized_checkpoint_getter(ck, qc)
    keys = set(ck.keys())
    out, n_q = {}, 0
    for k in ck.keys():
        if k.endswith((".qzeros", ".scales", ".g_idx", ".zp")) or ".quip_codes" in k:
            continue
        if k.endswith(".scale") and k[:-6] + ".weight" in keys:  # AutoRound native scale
            continue
        if k.endswith((".weight_scale", ".weight_scale_2", ".input_scale")):  # ModelOpt scales
            continue
        if k.endswith((".weight_blocks", ".weight_scales")):  # MXFP4: served under <name>.weight
            if k.endswith("_scales"):
                continue
            k = k[:-len("_blocks")]
            n_q += 1
        if k.endswith(".quip_scales"):
            name = k[:-len(".quip_scales")] + ".weight"
        else:
            name = k[:-8] + ".weight" if k.endswith(".qweight") else k
        v = get(name)
        if qc.get("quant_method") == "quip" and k.endswith(".quip_scales"):
            n_q += 1
        if k.endswith(".weight") and k + "_scale" in keys:  # ModelOpt NVFP4 / FP8 linear
            n_q += 1
        if isinstance(v, Int4Weight):
            v, n_q = v.dequantize(torch.float32), n_q + 1
        out[name] = v.to(torch.bfloat16) if v.is_floating_point() else v
    os.makedirs(args.dst, exist_ok=True)
    save_sharded(out, args.dst)
    hf.pop("quantization_config", None)
    hf["torch_dtype"] = "bfloat16"
    with open(os.path.join(args.dst, "config.json"), "w") as f:
        json.dump(hf, f, indent=1)
    for extra in ("tokenizer.json", "tokenizer_config.json", "generation_config.json", "special_tokens_map.json"):
        if os.path.exists(os.path.join(args.src, extra)):
            shutil.copy(os.path.join(args.src, extra), args.dst)
    print(f"wrote {args.dst}: {n_q} {qc['quant_method']} linears dequantized, {len(out)} tensors")


def cmd_show(args):
    if args.model.endswith(".gguf"):
        from .loaders.gguf import GGUFFile, GGML_TYPES, config_from_gguf
        f = GGUFFile(args.model)
        print(json.dumps(vars(config_from_gguf(f.metadata)), default=str, indent=1))
        for n, ti in list(f.tensors.items())[: args.max_tensors]:
            print(f"{n:48s} {GGML_TYPES[ti.ggml_type][0]:6s} {list(ti.shape)}")
        return
    from .engine.engine import load_model_source
    cfg, _, _ = load_model_source(args.model)
    print(json.dumps(vars(cfg), default=str, indent=1))
    print(f"parameters: {cfg.num_params() / 1e9:.2f} B")


def cmd_pull(args):
    from .utils import hub
    if args.verify:
        d = args.dest or os.path.join(os.environ.get("GOLLEK_HOME", os.path.expanduser("~/.gollek")), "models",
                                      args.repo_id)
        res = hub.verify(d)
        print(json.dumps(res, indent=1))
        if any(v != "ok" for v in res.values()):
            sys.exit(1)
        return
    d = hub.pull(args.repo_id, args.revision, args.dest, args.allow, args.endpoint)
    print(f"pulled {args.repo_id}@{args.revision} into {d}")


def cmd_list(args):
    from .config import PRESETS
    print("presets:")
    for k, v in PRESETS.items():
        print(f"  {k:16s} {v.num_params() / 1e9:7.2f} B params  {v.architecture}")
    home = os.environ.get("GOLLEK_HOME", os.path.expanduser("~/.gollek"))
    mdir = os.path.join(home, "models")
    if os.path.isdir(mdir):
        print(f"local models ({mdir}):")
        for n in sorted(os.listdir(mdir)):
            print("  " + n)


def cmd_transcribe(args):
    """Speech to text with a Whisper checkpoint: prints the text (or JSON with segments)."""
    import torch
    from .models.whisper import WhisperASR
    dev = args.device or ("cuda" if torch.cuda.is_available() else "cpu")
    asr = WhisperASR(args.model, device=dev, dtype=torch.float32 if dev == "cpu" else torch.bfloat16)
    datas = [open(f, "rb").read() for f in args.files]
    res = asr.transcribe(datas, language=args.language, task=args.task, timestamps=args.timestamps)
    for f, r in zip(args.files, res):
        if args.json:
            print(json.dumps({"file": f, **r}))
        else:
            print(r["text"])


def cmd_speak(args):
    """Text to speech with a SpeechT5 checkpoint and a HiFi-GAN vocoder: writes a 16-bit WAVE file."""
    import torch
    from .models.speecht5 import SpeechSynth
    dev = args.device or ("cuda" if torch.cuda.is_available() else "cpu")
    synth = SpeechSynth(args.model, args.vocoder, device=dev, dtype=torch.float32 if dev == "cpu" else torch.bfloat16)
    with open(args.out, "wb") as f:
        f.write(synth.wav_bytes(args.text, args.voice, args.seed))
    print(f"wrote {args.out}")


def cmd_bench(args):
    import subprocess
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.exit(subprocess.call([sys.executable, os.path.join(here, "bench.py")] + args.rest))


def build_parser():
    p = argparse.ArgumentParser(prog="gollek_b200")
    sub = p.add_subparsers(dest="cmd", required=True)

    def gen_opts(sp):
        sp.add_argument("--model", "-m", default="tiny-llama")
        sp.add_argument("--config", default=None)
        sp.add_argument("--device", default=None)
        sp.add_argument("--max-model-len", type=int, default=None)
        sp.add_argument("--max-tokens", type=int, default=128)
        sp.add_argument("--temperature", type=float, default=0.7)
        sp.add_argument("--top-p", type=float, default=0.95)
        sp.add_argument("--top-k", type=int, default=40)
        sp.add_argument("--seed", type=int, default=None)

    r = sub.add_parser("run")
    gen_opts(r)
    r.add_argument("prompt")
    r.add_argument("--stats", action="store_true")
    r.set_defaults(fn=cmd_run)
    c = sub.add_parser("chat")
    gen_opts(c)
    c.set_defaults(fn=cmd_chat)
    b = sub.add_parser("batch")
    gen_opts(b)
    b.add_argument("input")
    b.add_argument("output")
    b.set_defaults(fn=cmd_batch)
    s = sub.add_parser("serve", add_help=False)
    s.set_defaults(fn=cmd_serve)
    cv = sub.add_parser("convert")
    cv.add_argument("src")
    cv.add_argument("dst")
    gguf_types = ["F32", "F16", "BF16", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K",
                  "Q6_K", "Q3_K_M", "Q4_K_M", "Q5_K_M"]
    cv.add_argument("--type", default="F16", choices=gguf_types)
    cv.add_argument("--embed-type", default=None)
    cv.set_defaults(fn=cmd_convert)
    q = sub.add_parser("quantize")
    q.add_argument("src")
    q.add_argument("dst")
    q.add_argument("--type", default="Q4_K", help="GGUF source: target ggml type or mixture")
    q.add_argument("--method", default="fp8", choices=["fp8", "awq", "autoround", "quip", "nvfp4", "mxfp4"],
                   help="safetensors source: block-scaled fp8, AWQ or AutoRound int4 (calibrated), QuIP lattice")
    q.add_argument("--group", type=int, default=128, help="awq / autoround: input columns per scale")
    q.add_argument("--iters", type=int, default=200, help="autoround: signed-gradient steps per linear")
    q.add_argument("--stages", type=int, default=1, help="quip: 1 (2.25 bits per weight) or 2 (4.25)")
    q.add_argument("--calib-file", default=None, help="awq / autoround: token ids, one sequence per line")
    q.set_defaults(fn=cmd_quantize)
    dq = sub.add_parser("dequantize", help="GPTQ / AWQ / AutoRound / QuIP checkpoint -> dense bf16 safetensors")
    dq.add_argument("src")
    dq.add_argument("dst")
    dq.set_defaults(fn=cmd_dequantize)
    sh = sub.add_parser("show")
    sh.add_argument("model")
    sh.add_argument("--max-tensors", type=int, default=40)
    sh.set_defaults(fn=cmd_show)
    ls = sub.add_parser("list")
    ls.set_defaults(fn=cmd_list)
    pl = sub.add_parser("pull", help="download a hub repository (resumable, sha256-verified)")
    pl.add_argument("repo_id")
    pl.add_argument("--revision", default="main")
    pl.add_argument("--dest", default=None)
    pl.add_argument("--allow", nargs="*", default=None, help="file name patterns (default: serving files)")
    pl.add_argument("--endpoint", default=None)
    pl.add_argument("--verify", action="store_true", help="re-check an existing pull against its manifest")
    pl.set_defaults(fn=cmd_pull)
    tr = sub.add_parser("transcribe", help="speech to text (Whisper checkpoint, RIFF/WAVE input)")
    tr.add_argument("files", nargs="+")
    tr.add_argument("--model", "-m", required=True)
    tr.add_argument("--language", default=None, help="default: detected")
    tr.add_argument("--task", choices=["transcribe", "translate"], default="transcribe")
    tr.add_argument("--timestamps", action="store_true")
    tr.add_argument("--json", action="store_true")
    tr.add_argument("--device", default=None)
    tr.set_defaults(fn=cmd_transcribe)
    sp = sub.add_parser("speak", help="text to speech (SpeechT5 + HiFi-GAN checkpoints) into a WAV file")
    sp.add_argument("model")
    sp.add_argument("text")
    sp.add_argument("--vocoder", required=True)
    sp.add_argument("--out", default="speech.wav")
    sp.add_argument("--voice", default=None, help="speakers/<voice>.npy in the model directory")
    sp.add_argument("--seed", type=int, default=0)
    sp.add_argument("--device", default=None)
    sp.set_defaults(fn=cmd_speak)
    be = sub.add_parser("bench")
    be.add_argument("rest", nargs=argparse.REMAINDER)
    be.set_defaults(fn=cmd_bench)
    return p


def main(argv=None):
    from .utils.log import configure_logging
    configure_logging()
    args = build_parser().parse_args(argv)
    args.fn(args)


if __name__ == "__main__":
    main()
