"""One rank of the tensor-parallel parity check (launched by tests/test_gpu_tp.py under torch.distributed.run, one
process per GPU; host plumbing over gloo, the model's collectives over its own NCCL communicator).

Every rank builds its shard of the same seeded model and runs the same teacher-forced decode, then a few free steps.
Rank 0 gathers the logits slices, and checks: (1) the assembled logits against the FP64 oracle (bound 0.05 +
0.003|ref|) for the small shape; (2) against a one-device model with the same weights (TP vs TP-1: only the
summation order of the partial sums differs); (3) every rank chose the same free-run tokens, each the first argmax of
the assembled logits. Prints one JSON line and exits non-zero on failure."""
import argparse
import datetime
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

SMALL = dict(NAME="small", D_MODEL=256, LAYERS=2, HEADS=4, KV_HEADS=2, HEAD_DIM=64, FFN=512, VOCAB=1024,
             ROPE_THETA=1e6, EPS=1e-6, QKV_BIAS=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="small", choices=["small", "small8", "internlm7b"])
    ap.add_argument("--mode", default="fused", choices=["fused", "nccl", "two_shot"])
    args = ap.parse_args()
    import torch
    import torch.distributed as dist
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    from agxforge.inference import assemble, models
    from tests import modelcheck as MC

    if args.case == "internlm7b":
        shape, bits, B, cap, steps, check_oracle = models.INTERNLM25_7B.replace(LAYERS=2), 4, 32, 96, 3, False
    else:
        shape, bits, B, cap, steps, check_oracle = dict(SMALL), (8 if args.case == "small8" else 4), 32, 64, 4, True
    vocab = shape["VOCAB"] if isinstance(shape, dict) else shape.VOCAB
    cfg = dict(model=shape, bits=bits, batch=B, cap=cap, seed=9, keep_logits=True, tp=world, tp_rank=rank)
    m = assemble.build(dict(cfg), device=local, keep_packs=(rank == 0 and check_oracle))
    info = m.plan_info()["tp"]
    if args.mode == "nccl":
        m.set_option("tp_fused", 0)       # every rank sets the same value
    elif args.mode == "two_shot":
        m.set_option("tp_fused", 2)       # reduce-scatter + all-gather even with 2 ranks
    elif not info["fused_available"]:
        raise SystemExit("rank %d: the fused path is not available" % rank)
    rng = np.random.default_rng(21)
    prompts = [rng.integers(0, vocab, int(n)).tolist() for n in rng.integers(3, 30, B)]
    seqs, lg, _ = MC.run_forced(m, prompts, steps, seed=22)
    free_t, free_lg, _ = m.decode(3, want_tokens=True, want_logits=True)
    parts = [None] * world
    dist.all_gather_object(parts, (m.vocab_offset, lg, free_t, free_lg))
    ok, report = True, dict(case=args.case, world=world, rank=rank, mode=args.mode,
                            fused=m.plan_info()["tp"]["fused"], two_shot=m.plan_info()["tp"]["two_shot"])
    if rank == 0:
        parts.sort(key=lambda p: p[0])
        full = np.concatenate([p[1] for p in parts], axis=2)
        ffull = np.concatenate([p[3] for p in parts], axis=2)
        assert full.shape[2] == vocab
        # (3) identical free-run tokens on every rank, each the first argmax of the assembled logits
        for p in parts:
            ok &= bool(np.array_equal(p[2], parts[0][2]))
        ok &= all(int(free_t[i, b]) == int(np.argmax(ffull[i, b])) for i in range(3) for b in range(B))
        report["tokens_agree"] = bool(ok)
        # (2) against the one-device model with the same weights
        one = assemble.build(dict(cfg, tp=1, tp_rank=0), device=local)
        s1, lg1, _ = MC.run_forced(one, prompts, steps, seed=22)
        one.close()
        dmax = float(np.abs(full.astype(np.float64) - lg1).max())
        report["max_diff_vs_tp1"] = dmax
        ok &= dmax < 0.02
        # (1) against the FP64 oracle
        if check_oracle:
            rep = MC.compare(m, seqs, full, steps, which=[0, 7, B - 1])
            report["oracle"] = rep
        report["ok"] = bool(ok)
        print(json.dumps(report), flush=True)
    flag = [ok]
    dist.broadcast_object_list(flag, src=0)
    m.close()
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if flag[0] else 1)


if __name__ == "__main__":
    main()
