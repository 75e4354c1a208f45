"""Weight offload: layers streamed from pinned host memory give the tokens of resident weights."""
import pytest
import torch

from gollek_b200.config import EngineConfig, preset
from gollek_b200.engine.engine import LLMEngine
from gollek_b200.engine.sequence import SamplingParams
from gollek_b200.models.reference import init_random_weights


@pytest.mark.gpu
@pytest.mark.parametrize("n_off,depth", [(2, 1), (3, 2), (4, 3)])
def test_offload_matches_resident(n_off, depth):
    cfg = preset("tiny-llama")
    w = init_random_weights(cfg, seed=0)
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 70)]
    sp = SamplingParams(temperature=0.0, max_tokens=8, ignore_eos=True)
    outs = []
    for off in (0, n_off):
        ec = EngineConfig(device="cuda", max_num_seqs=4, max_num_batched_tokens=128, max_model_len=256,
                          offload_layers=off, offload_prefetch=depth)
        eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, num_blocks=64)
        outs.append([o.output_token_ids for o in eng.generate(prompts, sp)])
        if off:
            assert eng.model.offload is not None and eng.model.offload.bytes_copied > 0
            assert not eng.cfg.use_cuda_graphs
    assert outs[0] == outs[1]
