"""CPU stand-ins of the three expert-parallel device stages, built from the oracle.

They produce and consume exactly the buffers of the CUDA stages (record layout, rank-major token
order, ret_row, send counts), so the host orchestration in sonicmoe.ep -- count exchange, splits,
validation, the two all-to-alls -- runs on gloo ranks without a GPU.  Test infrastructure only.
"""
import numpy as np
import torch

from oracle import quant as oq
from oracle import routing as oroute
from oracle.layer import swiglu_interleaved
from sonicmoe.ep import DispatchState


def meta_offset(H):
    return (H + H // 128 + 15) // 16 * 16


def record_bytes(H, K):
    return (meta_offset(H) + 8 * K + 15) // 16 * 16


class FakeStages:
    def __init__(self, bad_count_rank=None, err_code_rank=None, err_code=0):
        self.bad_count_rank = bad_count_rank
        self.err_code_rank = err_code_rank  # this rank's expert stage reports err_code in its error word
        self.err_code = err_code
        self.rank = None

    def record_bytes(self, H, K):
        return record_bytes(H, K)

    def dispatch(self, x, logits, E, K, W, rank, sot, norm, err):
        self.rank = rank
        T, H = x.shape
        El = E // W
        rb = record_bytes(H, K)
        scores, idx = oroute.topk_route(logits.float().numpy(), K, sot, norm)
        q, sf = oq.quant_1x128(x.float().numpy())
        dests = idx // El
        first = np.zeros_like(idx, dtype=bool)
        for k in range(K):
            first[:, k] = ~np.any(dests[:, :k] == dests[:, k : k + 1], axis=1)
        records, ret_row = [], np.full(T * K, -1, dtype=np.int32)
        send_counts = np.zeros(W, dtype=np.int32)
        for d in range(W):
            for t in range(T):
                ks = np.nonzero(first[t] & (dests[t] == d))[0]
                if len(ks) == 0:
                    continue
                rec = np.zeros(rb, dtype=np.uint8)
                rec[:H] = q[t]
                rec[H : H + H // 128] = sf[t]
                mine = dests[t] == d
                loc = np.where(mine, idx[t] - d * El, -1).astype(np.int32)
                sc = np.where(mine, scores[t], 0).astype(np.float32)
                m = meta_offset(H)
                rec[m : m + 4 * K] = loc.view(np.uint8)
                rec[m + 4 * K : m + 8 * K] = sc.view(np.uint8)
                ret_row[t * K + ks[0]] = len(records)
                records.append(rec)
                send_counts[d] += 1
        if self.bad_count_rank == rank:
            send_counts[rank] = -5  # injected host-side fault (self slot, seen only here): caught before data moves
        s_max = T * min(K, W)
        buf = np.zeros((max(s_max, 1), rb), dtype=np.uint8)
        if records:
            buf[: len(records)] = np.stack(records)
        return DispatchState(T, K, logits, torch.from_numpy(scores), torch.from_numpy(idx), torch.from_numpy(buf),
                             torch.from_numpy(ret_row), torch.from_numpy(send_counts))

    def expert(self, records, R, H, I, El, K, w1, w2, err):
        if self.err_code_rank is not None and self.rank == self.err_code_rank:
            err[0] = self.err_code  # a device stage that gave up, made on the host
        rec = records.numpy()
        w1q, w1s = oq.quant_128x128(w1.float().numpy())
        w1d = torch.as_tensor(oq.dequant_128x128(w1q, w1s)).double()
        w2q, w2s = oq.quant_128x128(w2.float().numpy())
        w2d = torch.as_tensor(oq.dequant_128x128(w2q, w2s)).double()
        out = torch.zeros(R, H, dtype=torch.float64)
        freq = np.zeros(El, dtype=np.int32)
        G = H // 128
        for j in range(R):
            xd = torch.as_tensor(oq.dequant_1x128(rec[j : j + 1, :H], rec[j : j + 1, H : H + G])).double()[0]
            m = meta_offset(H)
            loc = rec[j, m : m + 4 * K].copy().view(np.int32)
            sc = rec[j, m + 4 * K : m + 8 * K].copy().view(np.float32)
            for k in range(K):
                e = int(loc[k])
                if e < 0:
                    continue
                freq[e] += 1
                a = swiglu_interleaved(w1d[e] @ xd)
                aq, as_ = oq.quant_1x128(a.float().numpy()[None])
                ad = torch.as_tensor(oq.dequant_1x128(aq, as_)).double()[0]
                out[j] += float(sc[k]) * (w2d[e] @ ad)
        return out.to(torch.bfloat16), torch.from_numpy(freq)

    def combine(self, ret, ret_row, T, K, H):
        out = torch.zeros(T, H, dtype=torch.float32)
        rr = ret_row.numpy()
        for t in range(T):
            for k in range(K):
                if rr[t * K + k] >= 0:
                    out[t] += ret[int(rr[t * K + k])].float()
        return out.to(torch.bfloat16)
