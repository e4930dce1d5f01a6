"""CPU stand-ins of the expert-parallel layer's steps, built on the oracle
(test infrastructure): the same interface as firepit_b200.ep.DeviceOps, on
CPU torch tensors, so the dispatch / combine logic runs with gloo ranks.

The expert MLP here is the f32 restatement y = W2[e] . SwiGLU(W1[e] . x) on
dequantized weights, row by row; it depends on nothing but the row and its
expert, so a correct dispatch gives the expert-parallel layer exactly the
single-rank result."""
import numpy as np
import torch

from oracle import oracle as O


class HostOps:
    def topk(self, logits, k, width):
        ids, w = O.moe_topk(logits.numpy(), k, width)
        return torch.from_numpy(ids), torch.from_numpy(w)

    def route_dest(self, ids, slots, per_rank):
        d = ids.numpy() // per_rank
        d[:, slots:] = 0
        return torch.from_numpy(np.ascontiguousarray(d, np.int32))

    def layout(self, ids, slots, experts, tile_rows, cap):
        tr, te, inv, rg, pad = O.moe_layout(ids.numpy(), slots, experts, tile_rows, cap)
        return dict(tr=torch.from_numpy(tr), te=torch.from_numpy(te), inv=torch.from_numpy(inv),
                    rg=torch.from_numpy(rg), pad=torch.tensor([pad], dtype=torch.int32))

    def route_meta(self, ids, inverse, slots, per_rank, rows):
        out = np.zeros(rows, np.int32)
        i, inv = ids.numpy(), inverse.numpy()
        for t in range(i.shape[0]):
            for s in range(slots):
                out[inv[t, s]] = i[t, s] % per_rank
        return torch.from_numpy(out)

    def gather(self, x, token_rows, rows):
        tr = token_rows.numpy()[:rows]
        xn = x.numpy()
        return torch.from_numpy(np.where((tr >= 0)[:, None], xn[np.maximum(tr, 0)], 0).astype(np.float32))

    def expert_mlp(self, x, local_e, w1, w2, per_rank, amax_reduce):
        amax_reduce(torch.zeros(1, dtype=torch.int32))  # the device path's two reductions, in order
        amax_reduce(torch.zeros(1, dtype=torch.int32))
        n, h = x.shape
        inter = w1.shape[0] // per_rank // 2
        xn = x.numpy()
        y = np.zeros((n, h), np.float32)
        for j in range(n):
            e = int(local_e[j])
            gu = w1[e * 2 * inter:(e + 1) * 2 * inter] @ xn[j]
            act = O.swiglu(gu.reshape(1, -1).astype(np.float32))[0]
            y[j] = w2[e * h:(e + 1) * h] @ act
        return torch.from_numpy(y)

    def combine(self, routed, inverse, weights, slots, out_dtype):
        return torch.from_numpy(O.moe_combine(routed.numpy(), inverse.numpy(), weights.numpy(), slots))
