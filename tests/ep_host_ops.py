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


class HostEpOps:
    """CPU stand-in of firepit_b200.ep.DeviceEpOps (the fixed-capacity
    layer): the same chunked records - one per (token, destination rank),
    tokens in order, the rest of each chunk marked empty - with f32 rows
    instead of NVFP4 codes.  A record row is [x (H) | local ids (width, -1
    where another rank owns the slot or the record is empty) | weights]."""

    def __init__(self, tokens, hidden, inter, experts, top_k, nranks, w1, w2):
        self.tokens, self.hidden, self.inter, self.experts, self.k, self.nranks = (tokens, hidden, inter, experts,
                                                                                   top_k, nranks)
        self.per_rank = experts // nranks
        self.width = 1 << (top_k - 1).bit_length()
        self.rows = nranks * tokens
        self.w1, self.w2 = w1, w2
        rec = hidden + 2 * self.width
        self.send = torch.zeros(self.rows, rec)
        self.recv = torch.zeros(self.rows, rec) if nranks > 1 else self.send
        self.ret_send = torch.zeros(self.rows, hidden)
        self.ret_recv = torch.zeros(self.rows, hidden) if nranks > 1 else self.ret_send

    def route(self, logits):
        ids, w = O.moe_topk(logits.numpy(), self.k, self.width)
        return torch.from_numpy(ids), torch.from_numpy(w)

    def amax(self, x):
        return torch.from_numpy(np.abs(x.numpy()).max(initial=0).astype(np.float32).reshape(1).view(np.int32))

    def dispatch(self, x, ids, w, amax):
        T, H, W, n, per = self.tokens, self.hidden, self.width, self.nranks, self.per_rank
        ids, w, xn = ids.numpy(), w.numpy(), x.numpy()
        send = np.zeros((self.rows, H + 2 * W), np.float32)
        pos = np.full(T * n + n, -1, np.int32)
        counts = [0] * n
        for t in range(T):
            owner = ids[t, :self.k] // per
            for d in range(n):
                if not np.any(owner == d):
                    continue
                r = d * T + counts[d]
                counts[d] += 1
                local = np.full(W, -1, np.int64)
                local[:self.k] = np.where(owner == d, ids[t, :self.k] % per, -1)
                send[r, :H] = xn[t]
                send[r, H:H + W] = local
                send[r, H + W:] = w[t]
                pos[t * n + d] = r
        for d in range(n):
            send[d * T + counts[d]:(d + 1) * T, H:H + W] = -1
        pos[T * n:] = counts
        self.send.copy_(torch.from_numpy(send))
        return self.send, torch.from_numpy(pos)

    def experts_gate_up(self, recv):
        H, W, I = self.hidden, self.width, self.inter
        r = recv.numpy()
        out = np.zeros((self.rows, H), np.float32)
        for j in range(self.rows):
            acc = np.zeros(H, np.float32)
            for s in range(self.k):
                e = int(r[j, H + s])
                if e < 0:
                    continue
                gu = self.w1[e * 2 * I:(e + 1) * 2 * I] @ r[j, :H]
                act = O.swiglu(gu.reshape(1, -1).astype(np.float32))[0]
                acc = acc + (self.w2[e * H:(e + 1) * H] @ act) * r[j, H + W + s]
            out[j] = acc
        self.ret_send.copy_(torch.from_numpy(out))
        return torch.zeros(1, dtype=torch.int32)

    def experts_down(self):
        return self.ret_send

    def finish(self, ret, pos):
        T, n = self.tokens, self.nranks
        rn, p = ret.numpy(), pos.numpy()[:T * n].reshape(T, n)
        out = np.zeros((T, self.hidden), np.float32)
        for t in range(T):
            for d in range(n):
                if p[t, d] >= 0:
                    out[t] = out[t] + rn[p[t, d]]
        return torch.from_numpy(out)
