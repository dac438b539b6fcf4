"""Worker for tests/test_gpu_cp_nccl.py: one process per GPU under torchrun.

Every rank builds the same seeded sequence, runs its span through
chunk_gdn2_cp with the NCCL all-gather, and checks outputs, the final state
and all gradients of its span against chunk_gdn2 run on the whole sequence on
its own GPU.  The same for the block's short convolution through
short_conv_cp (the W-1-row halo exchanged over NCCL, its gradient returned
to the previous rank; weight gradients all-reduced).  Exit status 0 means
every rank agreed.
"""

import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from qwendopamine_b200 import chunk_gdn2  # noqa: E402
from qwendopamine_b200.gdn2_ops.block_ops import short_conv  # noqa: E402
from qwendopamine_b200.gdn2_ops.cp import chunk_gdn2_cp, gather_span_maps, short_conv_cp  # noqa: E402


def rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30))


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    B, H, K, V = 1, 4, 128, 128
    T = 64 * 64 * world  # 64 chunks per rank: the span is cut into two sub-spans
    gen = torch.Generator(device=dev).manual_seed(0)
    bf = torch.bfloat16
    q = torch.randn(B, T, H, K, device=dev, generator=gen).to(bf)
    k = torch.randn(B, T, H, K, device=dev, generator=gen).to(bf)
    v = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
    # long memory (tiny decays, small erase gates) so the state entering a
    # span, and a sub-span, still matters thousands of tokens later
    g = -5e-4 * torch.rand(B, T, H, K, device=dev, generator=gen)
    b = (0.05 * torch.sigmoid(torch.randn(B, T, H, K, device=dev, generator=gen))).to(bf)
    w = torch.sigmoid(torch.randn(B, T, H, V, device=dev, generator=gen)).to(bf)
    h0 = torch.randn(B, H, K, V, device=dev, generator=gen) * 0.1
    do = torch.randn(B, T, H, V, device=dev, generator=gen).to(bf)
    dht = torch.randn(B, H, K, V, device=dev, generator=gen)
    names = ("q", "k", "v", "g", "b", "w")
    full = {n: t.clone().requires_grad_() for n, t in zip(names, (q, k, v, g, b, w))}
    hf = h0.clone().requires_grad_()
    o_ref, ht_ref = chunk_gdn2(*(full[n] for n in names), initial_state=hf,
                               output_final_state=True, use_qk_l2norm_in_kernel=True)
    ((o_ref.float() * do.float()).sum() + (ht_ref * dht).sum()).backward()
    span = T // world
    a, e = rank * span, (rank + 1) * span
    loc = {n: t[:, a:e].detach().clone().requires_grad_() for n, t in zip(names, (q, k, v, g, b, w))}
    hl = h0.clone().requires_grad_()
    o, ht = chunk_gdn2_cp(*(loc[n] for n in names), rank=rank, world=world,
                          gather=lambda t: gather_span_maps(t, None), initial_state=hl)
    loss = (o.float() * do[:, a:e].float()).sum()
    if rank == world - 1:
        loss = loss + (ht * dht).sum()
    loss.backward()
    errs = {"o": rel(o, o_ref[:, a:e])}
    if rank == world - 1:
        errs["ht"] = rel(ht, ht_ref)
    for n in names:
        errs["d" + n] = rel(loc[n].grad, full[n].grad[:, a:e])
    if rank == 0:
        errs["dh0"] = rel(hl.grad, hf.grad)
    # the block's short convolution, sequence-parallel
    D, W = 512, 4
    xc = torch.randn(2, T, D, device=dev, generator=gen).to(bf)
    wc = (torch.randn(D, 1, W, device=dev, generator=gen) * 0.5).to(bf)
    bc = (torch.randn(D, device=dev, generator=gen) * 0.5).to(bf)
    dyc = torch.randn(2, T, D, device=dev, generator=gen).to(bf)
    xf, wf, bff = (t.clone().requires_grad_() for t in (xc, wc, bc))
    yf, _ = short_conv(xf, wf, bff)
    (yf.float() * dyc.float()).sum().backward()
    xl = xc[:, a:e].clone().requires_grad_()
    wl, bl = wc.clone().requires_grad_(), bc.clone().requires_grad_()
    yl = short_conv_cp(xl, wl, bl, rank=rank, world=world,
                       gather=lambda t: gather_span_maps(t, None))
    (yl.float() * dyc[:, a:e].float()).sum().backward()
    dwl, dbl = wl.grad.float(), bl.grad.float()
    dist.all_reduce(dwl)
    dist.all_reduce(dbl)
    errs["conv_y"] = 0.0 if torch.equal(yl, yf[:, a:e]) else 1.0
    errs["conv_dx"] = rel(xl.grad, xf.grad[:, a:e])
    errs["conv_dw"] = rel(dwl, wf.grad.float())
    errs["conv_db"] = rel(dbl, bff.grad.float())
    # the spans are coupled: this rank's output differs from running its span
    # from a zero state (rank 0 has the global initial state, so check r > 0)
    if rank > 0:
        o0, _ = chunk_gdn2(*(loc[n].detach() for n in names), output_final_state=True,
                           use_qk_l2norm_in_kernel=True)
        errs["coupling"] = 0.0 if rel(o0, o_ref[:, a:e]) > 1e-2 else 1.0
    bad = {n: x for n, x in errs.items() if not x < 2e-2}
    print(f"rank {rank}: " + " ".join(f"{n}={x:.1e}" for n, x in errs.items()), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(1 if bad else 0)


if __name__ == "__main__":
    main()
