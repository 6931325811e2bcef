"""CPU restatement of the three compute steps of a sequence shard's forward (test
infrastructure only).

It reads and writes the same workspace regions as the native steps
(``lca_swa_shard_prepare`` / ``_forward`` / ``_finish``), at the offsets the native
library's own layout function returns, so that the exchange logic of
``long_context_attention.distributed`` can be run on ``gloo`` ranks without a GPU.  The
arithmetic is float64 numpy over the dense Longformer mask restricted to what a shard
holds: its own rows, the received halos and the exchanged compact global rows.
"""
from __future__ import annotations

import numpy as np
import torch

from long_context_attention.distributed import NativeShardSteps


def _region(ws: torch.Tensor, off: int, nbytes: int, dtype: torch.dtype) -> torch.Tensor:
    return ws[off:off + nbytes].view(dtype)


class CpuShardSteps:
    def __init__(self):
        self._native = NativeShardSteps()  # host-only layout function of the C ABI

    def layout(self, spec, num_unique_global):
        return self._native.layout(spec, num_unique_global)

    def workspace(self, nbytes, device):
        return torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=device)

    # ------------------------------------------------------------------ helpers
    def _dims(self, spec):
        return spec.batch * spec.heads, spec.head_dim

    def _globals(self, spec, lay, ws, dtype, G):
        bh, d = self._dims(spec)
        return _region(ws, lay.globals_offset, lay.globals_bytes, dtype).view(G, 3, bh, d)

    def _halo(self, spec, lay, ws, off, dtype):
        bh, d = self._dims(spec)
        h = lay.halo_rows
        return _region(ws, off, 2 * lay.halo_side_bytes, dtype).view(2, 2, bh, h, d)

    # ------------------------------------------------------------------ steps
    def prepare(self, spec, q, k, v, tokens, ws):
        lay = self.layout(spec, len(tokens))
        bh, d = self._dims(spec)
        G = len(tokens)
        n = spec.length
        if G:
            g = self._globals(spec, lay, ws, q.dtype, G)
            for j, t in enumerate(tokens):
                if spec.offset <= t < spec.offset + n:
                    r = t - spec.offset
                    for which, src in enumerate((q, k, v)):
                        g[j, which] = src.reshape(bh, n, d)[:, r]
        if lay.halo_rows:
            h = lay.halo_rows
            send = self._halo(spec, lay, ws, lay.halo_send_offset, q.dtype)
            for kv, src in enumerate((k, v)):
                s = src.reshape(bh, n, d)
                send[0, kv] = s[:, :h]
                send[1, kv] = s[:, n - h:]

    def forward(self, spec, q, k, v, out, lse, tokens, ws):
        lay = self.layout(spec, len(tokens))
        bh, d = self._dims(spec)
        G = len(tokens)
        n, off, N, w = spec.length, spec.offset, spec.seq_len, min(spec.window, spec.seq_len)
        f = lambda t: t.reshape(bh, -1, d).double().numpy()  # noqa: E731
        ql, kl, vl = f(q), f(k), f(v)
        # keys this shard can see: [off - h, off + n + h) from halo / local / halo
        h = lay.halo_rows
        lo_abs = max(0, off - h)
        hi_abs = min(N, off + n + h)
        kk = np.zeros((bh, hi_abs - lo_abs, d))
        vv = np.zeros((bh, hi_abs - lo_abs, d))
        kk[:, off - lo_abs:off - lo_abs + n] = kl
        vv[:, off - lo_abs:off - lo_abs + n] = vl
        if h:
            recv = self._halo(spec, lay, ws, lay.halo_recv_offset, q.dtype).double().numpy()
            if off > 0:
                kk[:, :off - lo_abs] = recv[0, 0][:, h - (off - lo_abs):]
                vv[:, :off - lo_abs] = recv[0, 1][:, h - (off - lo_abs):]
            if off + n < N:
                m = hi_abs - (off + n)
                kk[:, off + n - lo_abs:] = recv[1, 0][:, :m]
                vv[:, off + n - lo_abs:] = recv[1, 1][:, :m]
        gset = np.asarray(tokens, dtype=np.int64)
        if G:
            g = self._globals(spec, lay, ws, q.dtype, G).double().numpy()  # [G][3][bh][d]
            qg, kg, vg = (g[:, i].transpose(1, 0, 2) for i in range(3))
        o = np.zeros((bh, n, d))
        ls = np.zeros((bh, n))
        for i in range(n):
            a = off + i
            lo, hi = max(0, a - w), min(N - 1, a + w)
            keys = kk[:, lo - lo_abs:hi - lo_abs + 1]
            vals = vv[:, lo - lo_abs:hi - lo_abs + 1]
            if G:
                outside = (gset < lo) | (gset > hi)
                keys = np.concatenate([keys, kg[:, outside]], axis=1)
                vals = np.concatenate([vals, vg[:, outside]], axis=1)
            s = np.einsum("bd,bkd->bk", ql[:, i], keys) * spec.scale
            mx = s.max(axis=1, keepdims=True)
            p = np.exp(s - mx)
            l = p.sum(axis=1)
            o[:, i] = np.einsum("bk,bkd->bd", p, vals) / l[:, None]
            ls[:, i] = mx[:, 0] + np.log(l)
        out.copy_(torch.from_numpy(o.reshape(out.shape)).float())
        if lse is not None:
            lse.copy_(torch.from_numpy(ls.reshape(lse.shape)).float())
        if G:
            # this shard's partial for every global row over its own keys
            s = np.einsum("bgd,bkd->bgk", qg, kl) * spec.scale
            mx = s.max(axis=2, keepdims=True)
            p = np.exp(s - mx)
            l = p.sum(axis=2)
            po = np.einsum("bgk,bkd->bgd", p, vl) / l[..., None]
            pl = mx[..., 0] + np.log(l)
            rp = _region(ws, lay.rowpart_offset, lay.rowpart_bytes, torch.float32)
            rp[:bh * G * d] = torch.from_numpy(po.reshape(-1)).float()
            rp[bh * G * d:bh * G * (d + 1)] = torch.from_numpy(pl.reshape(-1)).float()

    def finish(self, spec, out, lse, tokens, ws):
        lay = self.layout(spec, len(tokens))
        G = len(tokens)
        if G == 0:
            return
        bh, d = self._dims(spec)
        world = spec.world_size
        allp = _region(ws, lay.rowpart_all_offset, world * lay.rowpart_bytes, torch.float32).double().numpy()
        allp = allp.reshape(world, -1)
        po = allp[:, :bh * G * d].reshape(world, bh, G, d)
        pl = allp[:, bh * G * d:bh * G * (d + 1)].reshape(world, bh, G)
        mx = pl.max(axis=0)
        wts = np.exp(pl - mx[None])
        o = (wts[..., None] * po).sum(axis=0) / wts.sum(axis=0)[..., None]
        ls = mx + np.log(wts.sum(axis=0))
        ov = out.view(bh, spec.length, d)
        lv = lse.view(bh, spec.length) if lse is not None else None
        for j, t in enumerate(tokens):
            if spec.offset <= t < spec.offset + spec.length:
                r = t - spec.offset
                ov[:, r] = torch.from_numpy(o[:, j]).float()
                if lv is not None:
                    lv[:, r] = torch.from_numpy(ls[:, j]).float()
