"""Helper run under torchrun by test_tp_gpu.py / test_tp_cpu.py: a TP=k
forward of a tiny model must match the single-rank forward of the same
(dummy-initialised) weights; the fused NVLink reduction must match a plain
sum of the ranks' partials."""

import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from swiftllm_b200.models.config import load_config  # noqa: E402
from swiftllm_b200.models.decoder import AttnMeta, DecoderModel  # noqa: E402
from swiftllm_b200.parallel.comm import build_tp_group, init_distributed  # noqa: E402


def meta(T, dev):
    nb = (T + 15) // 16
    return AttnMeta(num_seqs=1, num_decode_seqs=0, num_tokens=T, max_q_len=T, max_seq_len=T,
                    positions=torch.arange(T, dtype=torch.int32, device=dev),
                    slot_mapping=torch.arange(T, dtype=torch.int32, device=dev),
                    q_start=torch.tensor([0, T], dtype=torch.int32, device=dev),
                    seq_lens=torch.tensor([T], dtype=torch.int32, device=dev),
                    block_tables=torch.arange(nb, dtype=torch.int32, device=dev).view(1, nb),
                    logits_idx=torch.arange(T, dtype=torch.int32, device=dev))


def main():
    backend = sys.argv[1]          # "fused" | "nccl" | "gloo"
    name = sys.argv[2] if len(sys.argv) > 2 else "tiny-llama"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    cuda = backend != "gloo"
    if cuda:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        dev = torch.device("cuda", torch.cuda.current_device())
        dtype = torch.bfloat16
    else:
        dev, dtype = torch.device("cpu"), torch.float32
    init_distributed(rank, world, "nccl" if cuda else "gloo")
    cfg = load_config(name)
    tp = build_tp_group(rank, world, dev, "fused" if backend == "fused" else "nccl", cfg, 512)
    if backend == "fused":
        g = torch.Generator(device=dev).manual_seed(123 + rank)
        H = cfg.hidden_size
        for T in (1, 7, 256, 300):
            # plain all-reduce: sum of per-rank partials
            x = torch.randn(T, H, device=dev, generator=g).to(dtype)
            parts = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(parts, x)
            ref = torch.stack([p.float() for p in parts]).sum(0)
            got = tp.reduce(x.clone())
            torch.testing.assert_close(got.float(), ref, rtol=2e-2, atol=3e-2)
            # GEMM partial into the reduce buffer, then reduce + residual
            # shard + RMSNorm + all-gather in one kernel
            xa = torch.randn(T, 64, device=dev, generator=g).to(dtype)
            w = (torch.randn(H, 64, device=dev, generator=g) * 0.1).to(dtype)
            xs = [torch.empty_like(xa) for _ in range(world)]
            ws = [torch.empty_like(w) for _ in range(world)]
            dist.all_gather(xs, xa)
            dist.all_gather(ws, w)
            ref = sum(a.float() @ b.float().t() for a, b in zip(xs, ws))
            res = torch.randn(T, H, device=dev, generator=g).to(dtype)
            dist.broadcast(res, 0)
            nw = (torch.rand(H, device=dev, generator=g) + 0.5).to(dtype)
            dist.broadcast(nw, 0)
            r_ref = (ref.to(dtype).float() + res.float()).to(dtype).float()
            n_ref = r_ref * torch.rsqrt(r_ref.pow(2).mean(-1, keepdim=True) + 1e-5) * nw.float()
            from swiftllm_b200 import ops
            ops.linear(xa, w, out=tp.reduce_buffer(T, H))
            res_local = res.clone()
            got_n = tp.reduce_norm(T, res_local, nw, 1e-5)
            lo, hi = tp.shard(T)
            torch.testing.assert_close(got_n.float(), n_ref, rtol=3e-2, atol=3e-2)
            torch.testing.assert_close(res_local[lo:hi].float(), r_ref[lo:hi], rtol=2e-2, atol=3e-2)
            # vocab-parallel greedy: argmax and log-prob over the full vocabulary
            V = 1000
            lg = torch.randn(T, V, device=dev, generator=g)
            lg[0, 3 * rank + 1] = 50.0  # tie across ranks: the lowest index must win
            lgs = [torch.empty_like(lg) for _ in range(world)]
            dist.all_gather(lgs, lg)
            full = torch.cat(lgs, dim=-1)
            tok, lp = tp.vocab_greedy(lg, rank * V)
            want = full.argmax(-1)
            assert torch.equal(tok.long(), want), (tok[:4], want[:4])
            ref_lp = torch.log_softmax(full, -1).gather(1, want.view(-1, 1)).view(-1)
            torch.testing.assert_close(lp, ref_lp, rtol=1e-3, atol=1e-3)
            # fused all-gather of vocab-parallel fp32 logits: bit-identical to
            # NCCL's all_gather (twice, so a stale buffer would show)
            for _ in range(2):
                lv = torch.randn(T, cfg.vocab_size // world, device=dev, generator=g)
                lvs = [torch.empty_like(lv) for _ in range(world)]
                dist.all_gather(lvs, lv)
                assert torch.equal(tp.gather_vocab(lv), torch.cat(lvs, dim=-1))
        st = tp.C.read_status(True)
        assert st[0] == 0, st
    m = DecoderModel(cfg, dtype, dev, tp)
    m.allocate()
    m.init_dummy(0)
    full = DecoderModel(cfg, dtype, dev)
    full.allocate()
    full.init_dummy(0)
    T = 37
    ids = torch.randint(0, cfg.vocab_size, (T,), dtype=torch.int32, generator=torch.Generator().manual_seed(0)).to(dev)
    nb = (T + 15) // 16
    kv = torch.zeros(nb, cfg.num_layers, 2, m.local_kv_heads, 16, cfg.head_dim, dtype=dtype, device=dev)
    kv1 = torch.zeros(nb, cfg.num_layers, 2, full.local_kv_heads, 16, cfg.head_dim, dtype=dtype, device=dev)
    with torch.no_grad():
        a = m.compute_logits(m.forward(ids, meta(T, dev), kv))
        b = full.compute_logits(full.forward(ids, meta(T, dev), kv1))
    err = (a - b).abs().max().item()
    tol = 1e-3 if not cuda else 0.05 * b.abs().max().item() + 0.05
    assert err < tol, (err, tol)
    if backend == "fused":
        st = tp.C.read_status(True)
        assert st[0] == 0, st
    dist.barrier()
    if rank == 0:
        print("TP_OK", backend, name, world, err)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
