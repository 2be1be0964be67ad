"""CPU stand-ins for the kernel entry points of gpa_vggt_b200.kernels, built on
the oracle -- test infrastructure for exercising the host logic (model wiring,
frame sharding) on CPU.  install(monkeypatch_like) swaps them in."""
from types import SimpleNamespace

import torch

from oracle import gpa_oracle as O


def attention(q, k, v, bias, sm_scale, return_lse=False, out=None, status=None, combine=None,
              lse_out=None):
    b = None if bias is None else bias.reshape(bias.shape[0], bias.shape[1], 1, -1)
    o, lse = O.attention_keybias(q, k, v, b, sm_scale, return_lse=True)
    if combine is not None:                   # exact two-partition combine
        oa, la = combine
        mx = torch.maximum(la.double(), lse)
        wa, wb = torch.exp2(la.double() - mx), torch.exp2(lse - mx)
        o = O.lse_combine(oa, la.double(), o, lse)
        lse = mx + torch.log2(wa + wb)
    o, lse = o.to(q.dtype), lse.float()
    if lse_out is not None:
        lse_out.copy_(lse)
        lse, return_lse = lse_out, True
    if out is not None:
        out.copy_(o)
        o = out
    return (o, lse) if return_lse else o


def merge_roles(rand_idx, num_imgs, w, h, sx, sy, num_special, no_rand, device):
    mask = O.dst_mask(num_imgs, w, h, sx, sy, num_special,
                      None if rand_idx is None else rand_idx.cpu(), no_rand)
    dst, src = O.split_positions(mask)
    slot = torch.empty(mask.numel(), dtype=torch.int32)
    slot[dst] = torch.arange(dst.numel(), dtype=torch.int32)
    slot[src] = -torch.arange(src.numel(), dtype=torch.int32) - 1
    return dst.int(), src.int(), slot


def metric_split(metric, src_pos, dst_pos):
    m = O.normalize_rows(metric)
    return m[src_pos.long()].to(torch.bfloat16), m[dst_pos.long()].to(torch.bfloat16)


def sim_argmax(a, b, status=None):
    nms, nis = [], []
    for i in range(a.shape[0]):
        nm, ni, _ = O.sim_argmax(a[i], b[i])
        nms.append(nm.float())
        nis.append(ni.int())
    return torch.stack(nms), torch.stack(nis)


def merge_plan(node_max, node_idx, r, dst_pos, src_pos):
    """The oracle's plan, also in the CSR form of kernels.MergePlan."""
    from gpa_vggt_b200.kernels import MergePlan
    ns, nd = src_pos.numel(), dst_pos.numel()
    plan = O.merge_plan(node_max.double(), node_idx.long(), r, nd)
    merged = torch.nonzero(plan.merged).reshape(-1)
    ni = node_idx.long()
    seg_src = merged[torch.sort(ni[merged], stable=True).indices]
    seg_start = torch.zeros(nd + 1, dtype=torch.long)
    seg_start[1:] = torch.cumsum(torch.bincount(ni[merged], minlength=nd), 0)
    mp = MergePlan(ns, nd, int(merged.numel()), dst_pos, src_pos, plan.unm_src.int(), seg_start.int(),
                   seg_src.int(), plan.counts.float(), node_max, node_idx)
    mp.oracle, mp.dst, mp.src = plan, dst_pos.long(), src_pos.long()
    return mp


def merge_kv_rows(rows, src_map, dst_map, unm_src, seg_start, seg_src, num_dst, out, mean=True):
    r = rows.double()
    res = []
    for u in ([] if unm_src is None else unm_src.tolist()):
        res.append(r[int(src_map[u])])
    for j in range(num_dst):
        a0, a1 = int(seg_start[j]), int(seg_start[j + 1])
        acc = r[int(dst_map[j])].clone()
        for m in seg_src[a0:a1].tolist():
            acc = acc + r[int(src_map[m])]
        res.append(acc / (1 + a1 - a0) if mean else acc)
    out.copy_(torch.stack(res).to(out.dtype))
    return out


def merge_kv(t, plan, mean=True, out=None, log_counts=None):
    res = O.merge_heads(t, plan.oracle, plan.dst, plan.src, "mean" if mean else "sum").to(t.dtype)
    if out is not None:
        out.copy_(res)
        return out
    return res


def frame_pool(k, v, S, ph, pw, pts, kp):
    H, N, D = k.shape
    P = ph * pw + pts
    pk, pv, size, _ = O.frame_pool(k.reshape(H, S, P, D), v.reshape(H, S, P, D), ph, pw, pts, kp)
    return pk.to(k.dtype), pv.to(k.dtype), size


def lse_combine(oa, la, ob, lb, out=None):
    res = O.lse_combine(oa, la.double(), ob, lb.double()).to(oa.dtype)
    out.copy_(res)
    return out


def build_plan(metric, w, h, sx, sy, r, no_rand=False, generator=None, metric_dim=0,
               num_special=5, rand_idx=None, proj=None):
    N = metric.shape[0]
    S = N // (w * h + num_special)
    dst, src, _ = merge_roles(rand_idx, S, w, h, sx, sy, num_special, no_rand, metric.device)
    m = O.project_metric(metric.float(), proj.float(), autocast_bf16=False) if proj is not None else metric
    m = O.normalize_rows(m.float())
    nm, ni, _ = O.sim_argmax(m[src.long()], m[dst.long()])
    return merge_plan(nm, ni, r, dst, src)


def install(setattr_fn, fp32=True):
    """Swap the stand-ins into the kernel module (setattr_fn(obj, name, value))."""
    from gpa_vggt_b200 import kernels
    from gpa_vggt_b200.vggt import layers
    for name in ("attention", "merge_roles", "metric_split", "sim_argmax", "merge_plan", "merge_kv",
                 "merge_kv_rows", "frame_pool", "lse_combine"):
        setattr_fn(kernels, name, globals()[name])
    setattr_fn(layers, "build_plan", build_plan)
    if fp32:
        setattr_fn(layers, "BF16", torch.float32)
