"""The NCCL sequence-parallel layer on 2 GPUs against the single-GPU layer
(skipped unless two GPUs are visible)."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _main(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    from oracle import oracle
    from sgsa_b200 import ops, sp
    from sgsa_b200.inputs import CONFIGS, make_inputs_slice

    cfg = CONFIGS["b200_bf16"].scaled(name="spn", B=1, T=4096, H=2, top_k=300)
    full = make_inputs_slice(cfg, 0, cfg.T, seed=2, device="cuda")
    tl = cfg.T // world
    mine = {n: t[:, rank * tl:(rank + 1) * tl].contiguous() for n, t in full.items()}
    names = ("q", "k", "v", "beta", "gamma", "iq", "ik", "mix")
    out, st = sp.sp_layer_fwd(*(mine[n] for n in names), cfg.top_k, output_final_state=True)
    ref, st_ref = ops.sgsa_layer_fwd(*(full[n] for n in names), cfg.top_k, output_final_state=True)
    e_out = oracle.rel_l2(out.float().cpu().numpy(),
                          ref[:, rank * tl:(rank + 1) * tl].float().cpu().numpy())
    e_st = oracle.rel_l2(st.cpu().numpy(), st_ref.cpu().numpy())
    result[rank] = (e_out, e_st)
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sp_two_gpus_matches_single_gpu():
    result = mp.Manager().dict()
    mp.spawn(_main, args=(2, 29623, result), nprocs=2, join=True)
    for r in range(2):
        assert result[r][0] < 2e-3 and result[r][1] < 2e-3, dict(result)
