"""Expert parallelism across 2 GPUs of one box: routed experts split by rank
(contiguous ranges), one NVLink exchange per MoE layer, combine in ascending
expert id.  The logits of every rank must equal the single-GPU model's bit
for bit (the combine sums the same sequence), for a verify batch and for the
decodes after it.  Needs two GPUs; skipped otherwise."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG_ARGS = dict(hidden_size=1024, layer_count=3, head_count=8, q_lora_rank=256, expert_count=32,
                experts_per_token=8, moe_intermediate_size=256, vocab_size=4096, hash_layer_count=1,
                context=300, rows=4)
IDS = [3, 1000, 77, 2024]
DECODES = [5, 6, 7]


def _cfg():
    from floyd_b200 import CONFIGS, scaled
    return scaled(CONFIGS["c4_ds4_flash"], **CFG_ARGS)


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import floyd_b200
    cfg = _cfg()
    m = floyd_b200.Model(cfg, device=rank, seed=0, rank=rank, world=world)
    s = floyd_b200.Session(m, cfg["context"] + 32, 4)
    s.seed_context(cfg["context"], 7)
    handles = [None] * world
    dist.all_gather_object(handles, s.ep_handle())
    s.ep_connect(handles)
    dist.barrier()
    s.verify(IDS)
    rows = s.row_logits(4)
    dec = [s.decode(t) for t in DECODES]
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), rows=rows, dec=np.stack(dec))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpu_expert_parallel_equals_single_gpu(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    import floyd_b200
    port = 29500 + os.getpid() % 1000
    mp.spawn(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    cfg = _cfg()
    m = floyd_b200.Model(cfg, device=0, seed=0)
    s = floyd_b200.Session(m, cfg["context"] + 32, 4)
    s.seed_context(cfg["context"], 7)
    s.verify(IDS)
    rows = s.row_logits(4)
    dec = np.stack([s.decode(t) for t in DECODES])
    for r in range(2):
        got = np.load(tmp_path / f"rank{r}.npz")
        assert np.array_equal(got["rows"], rows), f"rank {r} verify rows"
        assert np.array_equal(got["dec"], dec), f"rank {r} decodes"
