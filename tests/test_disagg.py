"""Prefill/decode disaggregation and the cluster KV hand-off: a prefill engine computes prompts and
first tokens, the decode engine continues from the handed-off KV; outputs equal the oracle."""
import threading
import time

import pytest
import torch

from gollek_b200 import ops
from gollek_b200.cluster import (CacheHandoffRequest, HandoffClient, HandoffServer, NodeRole, RemoteHandoff,
                                 handoff_to_proto, proto_to_handoff)
from gollek_b200.config import EngineConfig
from gollek_b200.engine.disagg import DisaggregatedEngine
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.models.reference import ReferenceDecoder


def _engine(cfg, w, device="cpu", nb=96):
    ec = EngineConfig(device=device, dtype="float32" if device == "cpu" else "bfloat16", block_size=16,
                      max_num_seqs=8, max_num_batched_tokens=64, max_model_len=256, use_cuda_graphs=False)
    return LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=nb)


def _prompts(cfg):
    g = torch.Generator().manual_seed(21)
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 37, 70)]


def test_disaggregated_pair_matches_oracle(tiny_cfg, tiny_weights):
    prompts = _prompts(tiny_cfg)
    ref = ReferenceDecoder(tiny_cfg, tiny_weights)
    expect = [ref.greedy(p, 8)[0] for p in prompts]
    pd = DisaggregatedEngine(_engine(tiny_cfg, tiny_weights), _engine(tiny_cfg, tiny_weights, nb=64))
    outs = pd.generate(prompts, SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True))
    assert [o.output_token_ids for o in outs] == expect
    assert pd.handoffs == 3 and pd.handoff_bytes > 0
    assert pd.prefill.kv.num_free_blocks() == pd.prefill.num_blocks  # prefill side released everything


def test_handoff_wire_contract():
    f = CacheHandoffRequest.DESCRIPTOR.fields_by_name
    assert [f[n].number for n in ("request_id", "model_id", "prompt_token_count", "block_ids", "block_data",
                                  "metadata")] == [1, 2, 3, 4, 5, 6]
    assert CacheHandoffRequest.DESCRIPTOR.full_name == "tech.kayys.gollek.cluster.proto.CacheHandoffRequest"


def test_grpc_handoff_between_nodes(tiny_cfg, tiny_weights):
    prompts = _prompts(tiny_cfg)
    ref = ReferenceDecoder(tiny_cfg, tiny_weights)
    expect = [ref.greedy(p, 6)[0] for p in prompts]
    decode = _engine(tiny_cfg, tiny_weights, nb=64)
    server = HandoffServer("decode-0", NodeRole.DECODE).start()
    stop = threading.Event()
    finished = {}

    def decode_loop():  # the decode node's engine thread
        while not stop.is_set():
            server.drain(decode)
            if decode.has_unfinished():
                for o in decode.step():
                    if o.finished:
                        finished[o.request_id] = o.output_token_ids
            else:
                time.sleep(0.002)

    th = threading.Thread(target=decode_loop, daemon=True)
    th.start()
    try:
        client = HandoffClient(server.address)
        pong = client.ping("prefill-0")
        assert pong.role == "DECODE" and pong.ready and pong.node_id == "decode-0"
        prefill = _engine(tiny_cfg, tiny_weights)
        hook = RemoteHandoff(prefill, client)
        sp = SamplingParams(temperature=0.0, max_tokens=6, ignore_eos=True)
        ids = []
        for i, p in enumerate(prompts):
            rid = f"r{i}"
            hook.full_params[rid] = sp
            first = SamplingParams(**vars(sp))
            first.max_tokens = 1
            ids.append(prefill.add_request(rid, p, first))
        while prefill.has_unfinished():
            prefill.step()
        assert hook.sent == 3 and not hook.failed
        t0 = time.time()
        while len(finished) < 3 and time.time() - t0 < 60:
            time.sleep(0.01)
        assert [finished[i] for i in ids] == expect
    finally:
        stop.set()
        th.join(timeout=10)
        server.stop()


def test_handoff_proto_roundtrip(tiny_cfg, tiny_weights):
    from gollek_b200.engine.disagg import export_sequence
    eng = _engine(tiny_cfg, tiny_weights)
    eng.add_request("x", _prompts(tiny_cfg)[1], SamplingParams(temperature=0.0, max_tokens=1))
    seen = {}
    eng.handoff_hook = lambda s: seen.setdefault("h", export_sequence(eng, s)) is None
    while eng.has_unfinished():
        eng.step()
    h = seen["h"]
    back = proto_to_handoff(CacheHandoffRequest.FromString(handoff_to_proto(h).SerializeToString()))
    assert back.prompt_token_ids == h.prompt_token_ids and back.output_token_ids == h.output_token_ids
    torch.testing.assert_close(back.kv, h.kv, rtol=0, atol=0)


@pytest.mark.gpu
def test_kv_block_gather_scatter_gpu():
    L, NB, Hk, bs, D = 3, 40, 2, 16, 64
    cache = torch.randn(L, NB, 2, Hk, bs, D, device="cuda").bfloat16()
    ids = torch.tensor([5, 0, 39, 17], dtype=torch.int32, device="cuda")
    packed = ops.kv_gather_blocks(cache, ids)
    torch.testing.assert_close(packed, cache[:, ids.long()], rtol=0, atol=0)
    other = torch.zeros_like(cache)
    ops.kv_scatter_blocks(other, ids, packed)
    torch.testing.assert_close(other[:, ids.long()], cache[:, ids.long()], rtol=0, atol=0)
    assert float(other.float().abs().sum()) == float(cache[:, ids.long()].float().abs().sum())


@pytest.mark.gpu
def test_disaggregated_pair_gpu(tiny_cfg, tiny_weights):
    prompts = _prompts(tiny_cfg)
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    plain = _engine(tiny_cfg, tiny_weights, device="cuda").generate(prompts, sp)
    dev1 = "cuda:1" if torch.cuda.device_count() > 1 else "cuda"
    pre = _engine(tiny_cfg, tiny_weights, device="cuda")
    with torch.cuda.device(torch.device(dev1)):
        dec = _engine(tiny_cfg, tiny_weights, device="cuda")
    pd = DisaggregatedEngine(pre, dec)
    outs = pd.generate(prompts, sp)
    assert [o.output_token_ids for o in outs] == [o.output_token_ids for o in plain]
