"""GPU (two or more devices): split-KV decode across real GPUs, NCCL exchange and fused peer-memory exchange.

World-size 2 ranks (one process per GPU, NCCL) each hold only their own pages of one long
sequence (written through ``SplitKV.slot_mapping``).  ``SplitKV.attend`` (partial kernel,
NCCL all_gather, merge kernel) and ``SplitKV.attend_fused`` (the reader kernel stores its
partial into every rank's exchange buffer over NVLink and merges) must both equal the oracle's
unsplit attention on every rank.  Skipped on a one-GPU machine; the same logic is covered
there by tests/test_gpu_split_kv.py (emulated ranks) and tests/test_distributed_cpu.py (gloo).
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    from nvfp4_qsa import workloads as W
    return W.decode_config(seed=91, context=20000, topk=4096, page=3136, rows=2)


def _rank(rank, world, port, outdir):
    import torch.distributed as dist
    from nvfp4_qsa import distributed as D
    from nvfp4_qsa import kernels

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        case = _case()
        pages = (20000 + case.page - 1) // case.page
        sk = D.SplitKV(pages, case.page, world, rank)
        storage = torch.zeros(max(sk.local_blocks, 1), 2, case.page, 288, dtype=torch.uint8, device=dev)
        parts = storage.transpose(1, 2).split(144, dim=-1)
        kd, ks = parts[0].split((128, 16), dim=-1)
        vd, vs = parts[1].split((128, 16), dim=-1)

        def bits(a):
            return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)

        kernels.qsa_write_cache_nvfp4(bits(case.key), bits(case.value), kd, ks, vd, vs,
                                      sk.slot_mapping(torch.arange(20000, device=dev)), 1.0, 1.0)
        q = bits(case.query)
        idx = torch.from_numpy(case.indices).to(dev)
        t2r = torch.from_numpy(case.token_to_request).to(dev)
        nccl_out = torch.empty_like(q)
        sk.attend(q, kd, ks, vd, vs, 1.0, 1.0, idx, t2r, nccl_out)
        ex = D.PeerExchange(q.shape[0], 24, 2)
        fused = []
        for _ in range(3):  # both parities, re-armed
            out = torch.full_like(q, float("nan"))
            sk.attend_fused(q, kd, ks, vd, vs, 1.0, 1.0, idx, t2r, out, ex)
            fused.append(out)
        torch.cuda.synchronize()
        dist.barrier()
        ex.close()
        np.save(os.path.join(outdir, f"nccl_{rank}.npy"), nccl_out.float().cpu().numpy())
        for i, out in enumerate(fused):
            np.save(os.path.join(outdir, f"fused_{rank}_{i}.npy"), out.float().cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_split_kv_across_two_gpus_nccl_and_fused(tmp_path):
    import torch.multiprocessing as mp
    import oracle

    world = 2
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn", join=True)
    case = _case()
    storage = np.zeros((case.blocks, 2, case.page, 288), np.uint8)
    oracle.write_cache(case.key, case.value, storage, case.slots)
    expected = oracle.sparse_attention(case.query, storage, case.indices, case.block_table, case.token_to_request)
    from gpu_util import assert_attention_close
    for r in range(world):
        for name in [f"nccl_{r}"] + [f"fused_{r}_{i}" for i in range(3)]:
            got = torch.from_numpy(np.load(tmp_path / f"{name}.npy"))
            assert_attention_close(got, expected, name)
