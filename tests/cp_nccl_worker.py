"""Worker for tests/test_gpu_cp_nccl.py: one process per GPU under torchrun.

Every rank builds the same seeded sequence, runs its span through
chunk_gdn2_cp with the NCCL all-gather under a loss on its outputs and on its
returned end state, and checks the outputs, the end state and all gradients
of its span against (1) chunk_gdn2 chained over the spans on its own GPU and
(2) the float64 oracle on two heads of the whole sequence.  The same for the
block's short convolution through short_conv_cp (the W-1-row halo exchanged
over NCCL, its gradient returned to the previous rank; weight gradients
all-reduced), against the single-GPU convolution and the float64 oracle.
Exit status 0 means every rank agreed.
"""

import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from oracle import block_oracle as BO  # noqa: E402
from oracle import gdn2_oracle as O  # noqa: E402
from qwendopamine_b200 import chunk_gdn2  # noqa: E402
from qwendopamine_b200.gdn2_ops.block_ops import short_conv  # noqa: E402
from qwendopamine_b200.gdn2_ops.cp import chunk_gdn2_cp, gather_span_maps, short_conv_cp  # noqa: E402


def rel(a, b):
    return float((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30))


ORACLE_HEADS = (0, 3)


def oracle_errors(q, k, v, g, b, w, h0, do, dhts, o, ht, loc, a, e, span, world):
    """rel-L2 of this rank's outputs, end state and input gradients against
    the float64 oracle run on the whole sequence (two heads), with the loss
    on every span's end state routed as the reference chain routes it."""
    hs = list(ORACLE_HEADS)
    cpu = lambda t: t[:, :, hs].double().cpu().numpy()
    args = [cpu(t) for t in (q, k, v, g, b, w)]
    s0 = h0[:, hs].double().cpu().numpy()
    dh = dhts[:, :, hs].double().cpu().numpy()
    don = cpu(do)
    # forward: the state entering this span, then the span itself
    pre = [x[:, :a] for x in args]
    s_in = O.recurrent_fwd(*pre, s0, norm_mode="fla")[1] if a > 0 else s0
    ro, rh = O.recurrent_fwd(*(x[:, a:e] for x in args), s_in, norm_mode="fla")
    # backward: gradient of this span's end state from the later spans and
    # the direct terms, then this span's input gradients
    end = dh[world - 1]
    for j in range(world - 1, a // span, -1):
        sl = slice(j * span, (j + 1) * span)
        end = O.recurrent_bwd(*(x[:, sl] for x in args), don[:, sl], None, end,
                              norm_mode="fla")[-1] + dh[j - 1]
    ref = O.recurrent_bwd(*(x[:, a:e] for x in args), don[:, a:e], s_in, end, norm_mode="fla")
    relc = lambda x, r: rel(x.detach().cpu(), torch.from_numpy(r))
    out = {"o_oracle": relc(o[:, :, hs], ro), "ht_oracle": relc(ht[:, hs], rh)}
    for n, r in zip(("q", "k", "v", "g", "b", "w"), ref):
        out[f"d{n}_oracle"] = relc(loc[n].grad[:, :, hs], r)
    return out


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    B, H, K, V = 1, 4, 128, 128
    T = 128 * 64 * world  # 128 chunks per rank: the span is cut into four sub-spans
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
    # a distinct gradient for every rank's end state S_r: a loss on a middle
    # rank's returned state must reach that rank's and every earlier rank's
    # inputs
    dhts = torch.randn(world, B, H, K, V, device=dev, generator=gen)
    names = ("q", "k", "v", "g", "b", "w")
    span = T // world
    a, e = rank * span, (rank + 1) * span
    # reference on this GPU: the spans chained through chunk_gdn2 (each
    # span's end state is the next one's initial state), loss on every
    # output and every span's end state
    full = {n: t.clone().requires_grad_() for n, t in zip(names, (q, k, v, g, b, w))}
    hf = h0.clone().requires_grad_()
    state, o_parts, ht_parts, loss_ref = hf, [], [], 0.0
    for j in range(world):
        sl = slice(j * span, (j + 1) * span)
        o_j, state = chunk_gdn2(*(full[n][:, sl] for n in names), initial_state=state,
                                output_final_state=True, use_qk_l2norm_in_kernel=True)
        o_parts.append(o_j)
        ht_parts.append(state)
        loss_ref = loss_ref + (o_j.float() * do[:, sl].float()).sum() + (state * dhts[j]).sum()
    loss_ref.backward()
    o_ref = torch.cat(o_parts, 1)
    loc = {n: t[:, a:e].detach().clone().requires_grad_() for n, t in zip(names, (q, k, v, g, b, w))}
    hl = h0.clone().requires_grad_()
    o, ht = chunk_gdn2_cp(*(loc[n] for n in names), rank=rank, world=world,
                          gather=lambda t: gather_span_maps(t, None), initial_state=hl)
    loss = (o.float() * do[:, a:e].float()).sum() + (ht * dhts[rank]).sum()
    loss.backward()
    errs = {"o": rel(o, o_ref[:, a:e]), "ht": rel(ht, ht_parts[rank])}
    for n in names:
        errs["d" + n] = rel(loc[n].grad, full[n].grad[:, a:e])
    if rank == 0:
        errs["dh0"] = rel(hl.grad, hf.grad)
    # against the float64 oracle on two heads of the whole sequence: this
    # span's outputs, its end state and its input gradients
    errs.update(oracle_errors(q, k, v, g, b, w, h0, do, dhts, o, ht, loc, a, e, span, world))
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
    # the halo'd convolution against the float64 oracle of the whole sequence
    xo, wo, bo, dyo = (t.double().cpu().numpy() for t in (xc, wc[:, 0], bc, dyc))
    y_or = BO.conv_fwd(xo, wo, bo)
    dx_or = BO.conv_bwd(xo, wo, dyo, bias=bo)[0]
    errs["conv_y_oracle"] = rel(yl.detach().cpu(), torch.from_numpy(y_or[:, a:e]))
    errs["conv_dx_oracle"] = rel(xl.grad.cpu(), torch.from_numpy(dx_or[:, a:e]))
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
