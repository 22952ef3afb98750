"""Multi-GPU check run under torchrun by tests/test_ulysses_gpu.py (one process per GPU).

Every rank runs the hybrid block twice on identical seeded inputs: once on all
rows on its own GPU (no exchange), once sequence-sharded through the Ulysses
runtime (NCCL all-to-all around head-sharded attention, frame-sum all-reduce).
The rank's shard of the two outputs must agree: the GEMMs and producers are
row-independent and attention is head-independent, so the only difference is
the summation order of the frame mean that feeds alpha.  The same holds for
every branch-parallel layout (n softmax ranks + P - n VDA ranks, n = 1..P-1) and
for a packed sequence with text rows first and anchor frames (all-to-all exchange).
"""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from vdn_b200.block import BlockConfig, HybridBlock  # noqa: E402
from vdn_b200.ulysses import UlyssesRuntime, init_ulysses  # noqa: E402


@torch.no_grad()
def main():
    rt = init_ulysses("nccl", timeout_seconds=60)
    dev = rt.device
    failures = []
    branch_runtimes = {}
    for n_soft in range(1, rt.world_size):
        brt = UlyssesRuntime(rank=rt.rank, world_size=rt.world_size, local_rank=rt.local_rank,
                             device=dev, backend="nccl", timeout_seconds=60)
        brt.enable_branch_parallel(n_soft)
        branch_runtimes[n_soft] = brt
    text_rt = UlyssesRuntime(rank=rt.rank, world_size=rt.world_size, local_rank=rt.local_rank,
                             device=dev, backend="nccl", timeout_seconds=60, exchange_mode="alltoall")
    for frames, tokens in ((4, 64), (3, 100)):
        cfg = BlockConfig(hidden=512, heads=4, head_dim=128, ffn=1024, radius=1, lora_rank=8)
        block = HybridBlock(cfg, seed=3, device=dev)
        with torch.random.fork_rng(devices=[]):
            torch.manual_seed(11)
            torch.nn.init.normal_(block.softmax_gate.weight, std=0.05)
        g = torch.Generator().manual_seed(frames * 1000 + tokens)
        T = frames * tokens
        x = torch.randn(T, cfg.hidden, generator=g).bfloat16().to(dev)
        temb = torch.randn(cfg.hidden, generator=g).to(dev)
        full = block(x, temb, frames, tokens)
        rt.reset()
        rt.configure(T, cfg.heads)
        shards = {}
        for mode in ("alltoall", "peer", "peer"):     # the peer path twice: buffer reuse
            rt.exchange_mode = mode
            shard = block(x[rt.local_start:rt.local_end].contiguous(), temb, frames, tokens, rt)
            torch.cuda.synchronize()
            want = full[rt.local_start:rt.local_end].double()
            err = float((shard.double() - want).norm() / want.norm())
            ok = bool(torch.isfinite(shard).all()) and err < 2e-3
            print(f"rank {rt.rank} {mode} frames={frames} tokens={tokens} rows={shard.shape[0]} "
                  f"rel_l2={err:.3e}", flush=True)
            if not ok:
                failures.append((mode, frames, tokens, err))
            shards.setdefault(mode, shard)
            gathered = rt.gather_sequence(shard)
            if gathered.shape != full.shape:
                failures.append(("gather shape", tuple(gathered.shape)))
        # The peer path replayed from a CUDA graph (device-counter fences).
        from vdn_b200.block import BlockGraph
        local = x[rt.local_start:rt.local_end].contiguous()
        graph = BlockGraph(block, local, temb, frames, tokens, rt)
        for _ in range(2):
            out = graph.replay()
            torch.cuda.synchronize()
            if not torch.equal(out, shards["peer"]):
                d = (out.float() - shards["peer"].float()).abs().max().item()
                failures.append(("graph replay", frames, tokens, d))
        del graph
        for ex in rt._exchanges.values():
            ex.check()                              # no device fence timed out
        # Branch-parallel layouts: n softmax ranks + P - n VDA ranks.
        for n_soft, brt in branch_runtimes.items():
            brt.reset()
            brt.configure(T, cfg.heads)
            shard = block(x[brt.local_start:brt.local_end].contiguous(), temb, frames, tokens, brt)
            torch.cuda.synchronize()
            want = full[brt.local_start:brt.local_end].double()
            err = float((shard.double() - want).norm() / want.norm())
            ok = bool(torch.isfinite(shard).all()) and err < 2e-3
            print(f"rank {brt.rank} branch{n_soft}+{brt.world_size - n_soft} ({brt.branch_kind}) "
                  f"frames={frames} tokens={tokens} rows={shard.shape[0]} rel_l2={err:.3e}", flush=True)
            if not ok:
                failures.append((f"branch{n_soft}", frames, tokens, err))
        # Text rows packed first, anchor frames and the text seed through the all-to-all.
        L = 16
        tcfg = BlockConfig(hidden=512, heads=4, head_dim=128, ffn=1024, radius=1, lora_rank=8,
                           anchor_frames="both", text_state=True)
        tblock = HybridBlock(tcfg, seed=4, device=dev)
        with torch.random.fork_rng(devices=[]):
            torch.manual_seed(12)
            torch.nn.init.normal_(tblock.softmax_gate.weight, std=0.05)
        xt = torch.randn(L + T, tcfg.hidden, generator=g).bfloat16().to(dev)
        tfull = tblock(xt, temb, frames, tokens, text_rows=L)
        text_rt.reset()
        text_rt.configure(L + T, tcfg.heads)
        lo, hi = text_rt.local_start, text_rt.local_end
        shard = tblock(xt[lo:hi].contiguous(), temb, frames, tokens, text_rt, text_rows=L)
        torch.cuda.synchronize()
        want = tfull[lo:hi].double()
        err = float((shard.double() - want).norm() / want.norm())
        ok = bool(torch.isfinite(shard).all()) and err < 2e-3
        print(f"rank {rt.rank} text{L}+anchors frames={frames} tokens={tokens} rows={shard.shape[0]} "
              f"rel_l2={err:.3e}", flush=True)
        if not ok:
            failures.append(("text rows", frames, tokens, err))
        # The two exchanges move the same bytes: identical block outputs.
        if not torch.equal(shards["alltoall"], shards["peer"]):
            d = (shards["alltoall"].float() - shards["peer"].float()).abs().max().item()
            print(f"rank {rt.rank} alltoall vs peer max abs diff {d:.3e}", flush=True)
    # install_ulysses: the installed sharded model forward equals the unsharded stack.
    from vdn_b200.stack import HybridStack
    from vdn_b200.ulysses import install_ulysses
    scfg = BlockConfig(hidden=512, heads=4, head_dim=128, ffn=1024, radius=1, lora_rank=8)
    stack = HybridStack(scfg, depth=2, seed=5, device=dev)
    frames, tokens = 5, 48
    gs = torch.Generator().manual_seed(77)
    xs = torch.randn(frames * tokens, scfg.hidden, generator=gs).bfloat16().to(dev)
    ts = torch.randn(scfg.hidden, generator=gs).to(dev)
    want = stack(xs, ts, frames, tokens)
    irt = UlyssesRuntime(rank=rt.rank, world_size=rt.world_size, local_rank=rt.local_rank, device=dev,
                         backend="nccl", timeout_seconds=60)
    install_ulysses(stack, irt)
    got = stack(xs, ts, frames, tokens)
    torch.cuda.synchronize()
    err = float((got.double() - want.double()).norm() / want.double().norm())
    print(f"rank {rt.rank} install_ulysses depth=2 rows={got.shape[0]} rel_l2={err:.3e}", flush=True)
    if not (got.shape == want.shape and bool(torch.isfinite(got).all()) and err < 4e-3):
        failures.append(("install_ulysses", err))
    irt.close()
    rt.close()
    flag = torch.tensor([len(failures)], device=dev)
    dist.all_reduce(flag)
    dist.destroy_process_group()
    sys.exit(1 if int(flag.item()) else 0)


if __name__ == "__main__":
    main()
