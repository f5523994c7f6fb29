"""One rank of the slot-sharded RepEncoder check on several GPUs (launched by
tests/test_gpu_multi_gpu.py through torch.distributed.run; not a test module).

Workload: 28 slots x 20k bf16 rows, 96 users of 1..64 items, bag sizes
min(64, Zipf(1.5)) and ids Zipf(1.2) -- the large-vocabulary layout's
distributions at a size every rank can also hold whole.  Rank r keeps the
rows of the slots s with (s-1) % world == r.  For its item range every rank
checks, bit for bit:

* the NCCL all-to-all exchange == the exchange inside the pooling kernel
  (peer stores over NVLink into CUDA-IPC-mapped buffers, both buffers of the
  double-buffered pair) == the single-GPU fused forward (K1 + K2) on the
  whole table;
* the int8 activations, scales and bf16 output of up to 256 of its items ==
  the oracle (rsqrt of each row's variance taken on this GPU, as in ATen's
  CUDA LayerNorm).

Prints one JSON line per rank and exits non-zero if any check fails.
"""

import datetime
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)


def main() -> int:
    import torch
    import torch.distributed as dist

    from baidu_cti_grab_b200 import device_ops, sharding, synth
    from conftest import gpu_rsqrt
    from oracle import oracle as O
    from test_gpu_baseline_configs import _compact_sample

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    checks = {}
    try:
        cfg = synth.WorkloadConfig("slot-sharded-check", 20_000, "bfloat16", 96, 1, 64, "heavy64", 1.2)
        batch = synth.make_batch(cfg, seed=11)
        R = cfg.rows_per_slot
        bf = torch.bfloat16
        full = synth.make_table_torch(cfg.num_rows, seed=12, device=dev)  # same seed: the same table on every rank
        plan = sharding.make_slot_plan(rank, world, batch["user_offsets"])
        local_table = sharding.build_local_table(full, plan, R)
        gen = torch.Generator(device=dev).manual_seed(13)
        H = 28 * 512
        gamma = (1 + 0.1 * torch.randn(H, device=dev, generator=gen)).to(bf)
        beta = (0.05 * torch.randn(H, device=dev, generator=gen)).to(bf)
        w = torch.randn((512, H), device=dev, generator=gen) / H ** 0.5
        bias = (0.02 * torch.randn(512, device=dev, generator=gen)).to(bf)
        w_nk, w_scale = device_ops.quantize_weight_per_channel(w)
        values = [torch.from_numpy(batch[s][0]).to(dev) for s in range(1, 29)]
        offsets = [torch.from_numpy(batch[s][1]).to(dev) for s in range(1, 29)]

        def all_to_all(out, inp, out_splits, in_splits):
            dist.all_to_all_single(out, inp, out_splits, in_splits)

        enc = sharding.SlotShardedRepEncoder(plan, local_table, R, gamma, beta, 1e-5, w_nk, w_scale, bias,
                                             all_to_all=all_to_all)
        out_nccl = enc.forward(values, offsets)
        exchange = sharding.PeerExchange(plan, bf, dev, all_gather_object=(
            lambda obj: (lambda out: (dist.all_gather_object(out, obj), out)[1])([None] * world)))
        flag = torch.zeros(1, dtype=torch.float32, device=dev)
        outs_peer = [enc.forward_peer(values, offsets, exchange, lambda: dist.all_reduce(flag)).clone()
                     for _ in range(2)]
        torch.cuda.synchronize()
        dist.barrier()
        exchange.close()

        i0, i1 = plan.my_items
        sub = sharding.slice_items(batch, i0, i1)
        sv = [torch.from_numpy(sub[s][0]).to(dev) for s in range(1, 29)]
        so = [torch.from_numpy(sub[s][1]).to(dev) for s in range(1, 29)]
        q, scale, _, _ = device_ops.rep_gather_ln_quant(full, sv, so, gamma, beta, 1e-5)
        out_single = device_ops.w8a8_gemm(q, w_nk, scale, w_scale,
                                          torch.empty((i1 - i0, 512), dtype=bf, device=dev), bias=bias)
        checks["items"] = i1 - i0
        checks["nccl_equals_single_gpu"] = bool(torch.equal(out_nccl, out_single))
        checks["peer_equals_single_gpu"] = all(bool(torch.equal(o, out_single)) for o in outs_peer)

        m = min(i1 - i0, 256)
        host, osub = _compact_sample(torch, full, batch, i0, i0 + m)
        oq, osc = O.rep_forward(host, "bfloat16", osub, gamma.float().cpu().numpy(), beta.float().cpu().numpy(),
                                1e-5, rsqrt=gpu_rsqrt)
        ref = O.scaled_epilogue(O.gemm_i8_i32(oq, w_nk.cpu().numpy()), osc, w_scale.cpu().numpy(),
                                bias.float().cpu().numpy(), "bfloat16")
        checks["oracle_items"] = m
        checks["int8_equals_oracle"] = bool(np.array_equal(q[:m].cpu().numpy(), oq)) and \
            bool(np.array_equal(scale[:m].cpu().numpy(), osc))
        checks["output_equals_oracle"] = bool(np.array_equal(out_nccl[:m].float().cpu().numpy(), ref))
        checks["device_error"] = device_ops.device_error()
    finally:
        dist.barrier()
        dist.destroy_process_group()
    ok = all(v for k, v in checks.items() if k.endswith(("_gpu", "_oracle"))) and checks.get("device_error") == 0
    print(json.dumps({"rank": rank, "world": world, "ok": ok, **checks}), flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
