"""Rank body of the control-plane failure tests (spawned per rank, gloo on CPU)."""
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def _exit_now(q):
    """Abrupt process exit after flushing the result queue's feeder thread."""
    q.close()
    q.join_thread()
    os._exit(0)


def run(rank, world, port, scenario, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        from gollek_b200.config import EngineConfig, preset
        from gollek_b200.engine.engine import LLMEngine
        from gollek_b200.engine.sequence import SamplingParams
        from gollek_b200.models.reference import init_random_weights
        from gollek_b200.parallel.control import (ControlPlane, ControlTimeout, DriverEngine, ProtocolError,
                                                  RankFailure, follow)
        from gollek_b200.parallel.dist import NcclComm
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=20))
        store = dist.distributed_c10d._get_default_store()
        cp = ControlPlane(rank, world, store, timeout_s=4.0, heartbeat_s=0.2, stale_s=1.5).start_heartbeat()
        cfg = preset("tiny-llama")
        w = init_random_weights(cfg, seed=0)
        ec = EngineConfig(device="cpu", dtype="float32", block_size=16, max_num_seqs=4, max_num_batched_tokens=64,
                          max_model_len=256, use_cuda_graphs=False, tensor_parallel_size=world)
        eng = LLMEngine(ec, model_cfg=cfg, weights=w.__getitem__, comm=NcclComm(rank, world), num_blocks=64)
        sp = SamplingParams(temperature=0.0, max_tokens=5, ignore_eos=True)
        if rank == 0:
            drv = DriverEngine(eng, cp)
            if scenario in ("ok", "slow"):
                drv.add_request("a", list(range(1, 20)), sp)
                drv.add_request("b", list(range(5, 40)), sp)
                outs = {}
                while drv.has_unfinished():
                    for o in drv.step():
                        if o.finished:
                            outs[o.request_id] = o.output_token_ids
                drv.shutdown_workers()
                q.put((rank, "ok", outs))
            elif scenario == "rank_dies":
                drv.add_request("a", list(range(1, 30)), SamplingParams(temperature=0.0, max_tokens=50,
                                                                        ignore_eos=True))
                drv.step()
                drv.step()
                time.sleep(2.5)  # the worker exits after two steps; its heartbeat goes stale
                try:
                    drv.step()
                    q.put((rank, "no-failure", None))
                except RankFailure as e:
                    q.put((rank, "RankFailure", e.rank))
                cp.stop()
                _exit_now(q)  # peers are gone: skip process-group teardown
            elif scenario == "drop":
                drv.add_request("a", list(range(1, 20)), sp)
                drv.step()  # step 1 published and run; step 2 is "dropped": never published
                time.sleep(6.0)
                q.put((rank, "driver-done", None))
                cp.stop()
                _exit_now(q)
            elif scenario == "corrupt":
                cp.store.set("step/1", b"\x00\x01garbage")
                time.sleep(3.0)
                q.put((rank, "driver-done", None))
                cp.stop()
                _exit_now(q)
        else:
            if scenario == "rank_dies":
                follow(eng, cp, max_steps=2)
                q.put((rank, "exiting", None))
                _exit_now(q)  # abrupt death between steps: no heartbeat stop, no teardown
            if scenario == "slow":
                orig = eng.step

                def slow_step():
                    time.sleep(0.5)  # a slow rank within every timeout
                    return orig()
                eng.step = slow_step
            try:
                n = follow(eng, cp)
                q.put((rank, "ok", n))
            except ControlTimeout:
                q.put((rank, "ControlTimeout", None))
            except ProtocolError as e:
                q.put((rank, "ProtocolError", str(e)))
            except RankFailure as e:
                q.put((rank, "RankFailure", e.rank))
            if scenario in ("drop", "corrupt"):
                cp.stop()
                _exit_now(q)
        cp.stop()
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        import traceback
        q.put((rank, "error", traceback.format_exc()))
