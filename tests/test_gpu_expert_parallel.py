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


@pytest.mark.parametrize("head_shard", ["0", "1"])
def test_two_gpu_expert_parallel_equals_single_gpu(tmp_path, monkeypatch, head_shard):
    """head_shard "1": each rank also runs half the attention heads and
    hands its W_UV outputs to the peer (FLOYD_HEAD_SHARD=1); the results
    stay bit-identical to one GPU either way."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    monkeypatch.setenv("FLOYD_HEAD_SHARD", head_shard)
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


def _batch_rank_main(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import floyd_b200
    cfg = _cfg()
    m = floyd_b200.Model(cfg, device=rank, seed=0, rank=rank, world=world)
    bs = floyd_b200.BatchSession(m, cfg["context"] + 32, 3, 4, 64)
    handles = [None] * world
    dist.all_gather_object(handles, bs.ep_handle())
    bs.ep_connect(handles)
    dist.barrier()
    _seed_batch(bs)
    n, nxt = bs.verify_batch(BATCH_IDS)
    np.savez(os.path.join(out_dir, f"batch{rank}.npz"), n=np.array(n), nxt=np.array(nxt), rows=bs.row_logits(4))
    dist.barrier()
    dist.destroy_process_group()


BATCH_IDS = [[3, 1000, 77, 2024], [5, 6, 7, 8], [11, 12, 13, 14]]


def _seed_batch(bs):
    bs.seed(0, 0, 64, 7)
    for q in range(3):
        bs.seed(q, 64, 150 + 40 * q, 100 + q)


def test_two_gpu_batch_verify_equals_single_gpu(tmp_path):
    """The batched multi-sequence verify over expert parallelism: every
    rank's commits, next tokens and last-pass rows equal one GPU's."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    import floyd_b200
    port = 29600 + os.getpid() % 1000
    mp.spawn(_batch_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    cfg = _cfg()
    m = floyd_b200.Model(cfg, device=0, seed=0)
    bs = floyd_b200.BatchSession(m, cfg["context"] + 32, 3, 4, 64)
    _seed_batch(bs)
    n, nxt = bs.verify_batch(BATCH_IDS)
    rows = bs.row_logits(4)
    for r in range(2):
        got = np.load(tmp_path / f"batch{r}.npz")
        assert got["n"].tolist() == n and got["nxt"].tolist() == nxt, f"rank {r}"
        assert np.array_equal(got["rows"], rows), f"rank {r} rows"


def _skip_rank_main(rank, world, port, out_dir):
    """Rank 1 stays alive but skips one forward call (between steps, with
    nothing of its own in flight); rank 0's combine waits for rank 1's epoch
    flag, gives up after its bounded wait and reports it.  Then both ranks
    rebuild their sessions (fresh receive regions and epoch flags), reconnect
    and verify again."""
    import time

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import floyd_b200
    cfg = _cfg()
    m = floyd_b200.Model(cfg, device=rank, seed=0, rank=rank, world=world)

    def connected_session():
        s = floyd_b200.Session(m, cfg["context"] + 32, 4)
        s.seed_context(cfg["context"], 7)
        handles = [None] * world
        dist.all_gather_object(handles, s.ep_handle())
        s.ep_connect(handles)
        dist.barrier()
        return s

    s = connected_session()
    s.verify(IDS)
    dist.barrier()
    result = {}
    if rank == 0:
        t0 = time.time()
        try:
            s.verify(IDS)
            result["error"] = ""
        except floyd_b200.FloydError as exc:
            result["error"] = str(exc)
        result["seconds"] = time.time() - t0
    dist.barrier()  # rank 1 skipped that forward
    s.close()
    s = connected_session()
    s.verify(IDS)
    np.savez(os.path.join(out_dir, f"skip{rank}.npz"), rows=s.row_logits(4),
             error=np.array(result.get("error", "")), seconds=np.array(result.get("seconds", 0.0)))
    dist.barrier()
    s.close()
    dist.destroy_process_group()


def test_two_gpu_rank_that_skips_a_forward_is_detected_and_recovered(tmp_path):
    """Failure detection without a GPU fault: the bounded epoch-flag wait of
    the expert exchange runs out (about 1 s per MoE layer) and the verify on
    the waiting rank returns "a kernel wait gave up"; after both ranks
    reconnect fresh sessions the results equal one GPU's again."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    import floyd_b200
    port = 29700 + os.getpid() % 1000
    mp.spawn(_skip_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    got0 = np.load(tmp_path / "skip0.npz")
    assert "gave up" in str(got0["error"]), str(got0["error"])
    moe_layers = CFG_ARGS["layer_count"]  # every layer of this config has experts
    assert float(got0["seconds"]) < 2.0 * moe_layers + 5.0
    cfg = _cfg()
    m = floyd_b200.Model(cfg, device=0, seed=0)
    s = floyd_b200.Session(m, cfg["context"] + 32, 4)
    s.seed_context(cfg["context"], 7)
    s.verify(IDS)
    rows = s.row_logits(4)
    for r in range(2):
        got = np.load(tmp_path / f"skip{r}.npz")
        assert np.array_equal(got["rows"], rows), f"rank {r} after recovery"
