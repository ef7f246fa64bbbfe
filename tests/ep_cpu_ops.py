"""A CPU stand-in for aero_b200.ep.CudaEpOps, for testing the expert-parallel
host protocol (splits, exchange order, reverse exchange, combine order) over
gloo without a GPU. Same buffer contracts as the C ABI entry points
aero_cuda_ep_dispatch / _expert_block / _combine; the arithmetic comes from the
oracle (test infrastructure only)."""

import numpy as np
import torch

import oracle as O


def _silu(v):
    return v / (1.0 + np.exp(-v))


class CpuEpOps:
    def __init__(self, layer, e_begin: int, e_end: int):
        sp = layer.spec
        self.layer, self.sp = layer, sp
        self.e_begin, self.e_end = e_begin, e_end
        self.meta_ld = 2 * sp.k + 2
        n_gu, n_dn = sp.F * sp.d, sp.d * sp.F
        bpe = lambda raw, n: raw.size // sp.E  # bytes per expert
        g, u, dn = (np.asarray(v).reshape(-1) for v in (layer.gate, layer.up, layer.down))
        self.W = {}
        for e in range(e_begin, e_end):
            sl = lambda raw: raw[e * bpe(raw, 0):(e + 1) * bpe(raw, 0)]
            self.W[e] = (O.dequant(sp.dtype, sl(g), n_gu).reshape(sp.F, sp.d),
                         O.dequant(sp.dtype, sl(u), n_gu).reshape(sp.F, sp.d),
                         O.dequant(sp.dtype, sl(dn), n_dn).reshape(sp.d, sp.F))
        sh = layer.shexp
        self.S = None
        if sh:
            fs = sh["ffn_len"]
            self.S = (O.dequant(sh["dtype"], sh["gate"], fs * sp.d).reshape(fs, sp.d),
                      O.dequant(sh["dtype"], sh["up"], fs * sp.d).reshape(fs, sp.d),
                      O.dequant(sh["dtype"], sh["down"], sp.d * fs).reshape(sp.d, fs),
                      np.asarray(sh["gate_inp"], np.float32).reshape(-1))

    def set_stream(self, stream):
        pass

    @staticmethod
    def _ffn(W, x):
        g, u, d = W
        return d @ (_silu(g @ x) * (u @ x))

    def dispatch(self, x, T, world, rank, begin, row_dtype, self_rows, self_meta, send_rows, send_meta, counts, pos):
        sp, k = self.sp, self.sp.k
        xn = x.numpy()
        lg = O.router_logits(xn, self.layer.router, self.layer.router_bias)
        idx, w = O.route(lg, k, sp.norm_topk_prob) if T else (np.zeros((0, k), np.int64), np.zeros((0, k), np.float32))
        sg = np.zeros(T, np.float32)
        if self.S is not None and T:
            sg = (1.0 / (1.0 + np.exp(-(xn @ self.S[3])))).astype(np.float32)
        rows_np = lambda t: torch.from_numpy(xn[t]).to(self_rows.dtype)

        def meta(t, dst, self_row):
            m = np.zeros(self.meta_ld, np.int32)
            lo, hi = begin[dst], begin[dst + 1]
            m[:k] = np.where((idx[t] >= lo) & (idx[t] < hi), idx[t], -1)
            m[k:2 * k] = w[t].view(np.int32)
            m[2 * k] = np.float32(sg[t] if self_row else 0.0).view(np.int32)
            return torch.from_numpy(m)

        for t in range(T):
            self_rows[t] = rows_np(t)
            self_meta[t] = meta(t, rank, True)
        slab = send_rows.shape[0] // world
        cnt = [0] * world
        pos_np = np.full((max(T, 1), world), -1, np.int32)
        pad = np.zeros(self.meta_ld, np.int32)
        pad[:k] = -1
        for r in range(world):
            for t in range(T):
                if r == rank:
                    pos_np[t, r] = t
                    continue
                if np.any((idx[t] >= begin[r]) & (idx[t] < begin[r + 1])):
                    row = r * slab + cnt[r]
                    send_rows[row] = rows_np(t)
                    send_meta[row] = meta(t, r, False)
                    pos_np[t, r] = row
                    cnt[r] += 1
            for j in range(cnt[r], slab):  # padding rows name no expert
                send_meta[r * slab + j] = torch.from_numpy(pad)
        counts[:world] = torch.tensor(cnt, dtype=torch.int32)
        counts[world] = sum(cnt)
        pos[:max(T, 1)] = torch.from_numpy(pos_np)

    def expert_block(self, rows, row_dtype, meta, R, n_shared, out):
        k = self.sp.k
        for r in range(R):
            xr = rows[r].float().numpy().astype(np.float32)
            m = meta[r].numpy()
            acc = np.zeros(self.sp.d, np.float32)
            for s in range(k):
                e = int(m[s])
                if e < 0:
                    continue
                assert self.e_begin <= e < self.e_end
                acc += np.float32(m[k + s:k + s + 1].view(np.float32)[0]) * self._ffn(self.W[e], xr)
            if r < n_shared and self.S is not None:
                acc += m[2 * k:2 * k + 1].view(np.float32)[0] * self._ffn(self.S[:3], xr)
            out[r] = torch.from_numpy(acc.astype(np.float32))

    def combine(self, self_out, back, pos, T, world, rank, out):
        for t in range(T):
            acc = self_out[t].clone()
            for r in range(world):
                p = int(pos[t, r])
                if r != rank and p >= 0:
                    acc += back[p]
            out[t] = acc
