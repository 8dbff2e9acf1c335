"""Run by tests/test_block_gpu.py under torchrun (2 ranks, one GPU each): the token-sharded DiT block with the ring and
the all-gather key/value exchanges (in head groups, and all at once) and the overlapped point-to-point exchange
against the unsharded block on rank 0's GPU.  Prints RING_OK / GATHER_OK / GATHER1_OK / OVERLAP_OK."""
import os
import sys
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
import conftest  # noqa: E402,F401
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from minimax_h3_turbo_b200.h3 import block as blk  # noqa: E402
from minimax_h3_turbo_b200.h3.synth import synthetic_activation, synthetic_w4a8  # noqa: E402
from minimax_h3_turbo_b200.h3.types import BlockWeights  # noqa: E402

HID, HEADS, HD, FFN, S = 512, 4, 128, 1024, 777


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        g = torch.Generator(device=dev).manual_seed(0)
        w = BlockWeights(qkv=synthetic_w4a8(3 * HID, HID, seed=1, device=dev), out=synthetic_w4a8(HID, HID, seed=2, device=dev),
                         fc1=synthetic_w4a8(2 * FFN, HID, seed=3, device=dev), fc2=synthetic_w4a8(HID, FFN, seed=4, device=dev),
                         norm1=(1 + 0.1 * torch.randn(HID, generator=g, device=dev)).bfloat16(),
                         norm2=(1 + 0.1 * torch.randn(HID, generator=g, device=dev)).bfloat16(),
                         q_norm=(1 + 0.1 * torch.randn(HD, generator=g, device=dev)).bfloat16(),
                         k_norm=(1 + 0.1 * torch.randn(HD, generator=g, device=dev)).bfloat16())
        mod = blk.Modulation(*(torch.randn(2, HID, generator=g, device=dev).bfloat16() for _ in range(6)))
        x = synthetic_activation(S, HID, seed=7, device=dev)
        pos = blk.video_audio_positions(7, 10, 10, S - 700, dev)
        cos, sin = blk.rope_tables(pos, 1.0 / (10000 ** (torch.arange(16, device=dev) / 16)), torch.bfloat16)
        segs_full = [(0, 700, 0), (700, S, 1)]
        ref = blk.DiTBlock(HEADS, HD)(x.clone(), w, mod, segs_full, cos, sin)
        a, b = blk.shard_rows(S, world, rank)
        spec = blk.ShardSpec(a, b, S, dist.group.WORLD, world, rank)
        segs = [(max(s0, a) - a, min(s1, b) - a, r) for s0, s1, r in segs_full if min(s1, b) > max(s0, a)]
        # gather: K/V all-gathered in 4 head groups (one head each here); gather1: all heads at once
        for mode, exchange, groups in (("ring", "ring", 1), ("gather", "gather", 4), ("gather1", "gather", 1),
                                       ("overlap", "overlap", 1)):
            block = blk.DiTBlock(HEADS, HD, kv_exchange=exchange, kv_groups=groups)
            y = block(x[a:b].clone(), w, mod, segs, cos[a:b], sin[a:b], spec)
            full = blk.gather_rows(y, spec)
            upd, want = full.float() - x.float(), ref.float() - x.float()
            rel = ((upd - want).norm() / want.norm()).item()
            ok = torch.isfinite(full.float()).all().item() and rel < 3e-2
            if rank == 0:
                print(f"{mode.upper()}_{'OK' if ok else 'BAD'} rel={rel:.3e}", flush=True)
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
