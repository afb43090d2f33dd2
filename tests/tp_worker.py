"""Worker for the tensor-parallel GPU test: one process per GPU (torch.multiprocessing spawn).

Every rank builds the same seeded model, runs it once on its own GPU without tensor parallelism,
once with the FeedForward / out_proj split over all ranks (NCCL) and once with the whole mixer split
too (SISO channel-parallel, MIMO head-parallel), and checks that the logits of prefill and of three greedy decode
steps are bit-identical.  Rank 0 writes the verdict."""
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def run(rank, world, port, out_path, cfg_kw, batch, seqlen):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from helpers import build_model
    from tesm_b200 import parallel
    model = build_model(cfg_kw).cuda().to(torch.bfloat16)
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, cfg_kw["vocab_size"], (batch, seqlen), generator=g).cuda()

    def run_model():
        with torch.no_grad():
            ip = {"state_cache": model.backbone.allocate_inference_cache(batch, seqlen + 8)}
            out, _ = model(ids, inference_params=ip, logits_to_keep=1)
            logits = [out.logits[:, -1].float().clone()]
            tok = out.logits[:, -1].argmax(-1, keepdim=True)
            for _ in range(3):
                o, _ = model(tok, inference_params=ip, logits_to_keep=1)
                logits.append(o.logits[:, -1].float().clone())
                tok = o.logits[:, -1].argmax(-1, keepdim=True)
        return torch.stack(logits)

    ref = run_model()
    parallel.enable_tensor_parallel(model)
    tp = run_model()
    # the sharded path really ran: every block holds its FFN and out_proj shards
    used = all("_b200_tp_shards" in b.mlp.__dict__ and "_b200_tp_out" in b.mixer.__dict__
               for b in model.backbone.layers)
    # then the whole SISO layer channel-parallel as well (in_proj by segment, channel-sharded
    # scan / window / decode cache, all-gathers, column-parallel combine, row-parallel out_proj)
    parallel.enable_mixer_parallel(model)
    mix = run_model()
    used_mix = all(("_b200_tp_mix" in b.mixer.__dict__ or "_b200_tp_mimo" in b.mixer.__dict__)
                   for b in model.backbone.layers)
    same = torch.equal(ref, tp) and used and torch.equal(ref, mix) and used_mix
    diff = (ref - tp).abs().max().item()
    diff_mix = (ref - mix).abs().max().item()
    ok = torch.tensor([1 if same else 0], device="cuda")
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    used = used and used_mix
    diff = max(diff, diff_mix)
    if rank == 0:
        with open(out_path, "w") as f:
            json.dump({"bit_identical": bool(ok.item()), "sharded_path_used": used, "max_abs_diff_rank0": diff,
                       "world": world}, f)
    dist.barrier()
    dist.destroy_process_group()
