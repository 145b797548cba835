"""Decode the Sage workspace (codes and scales written by the GPU) into logical arrays."""
import numpy as np

from oracle.sage import unswizzle_tile


def region(ws_np: np.ndarray, offs, i):
    return ws_np[offs[i]:offs[i + 1]]


def decode(ws_np, offs, batch, Hq, Hkv, lens_q, lens_k, tile0_q, tile0_k):
    """Returns per (b, h) dicts with qcodes/qscales (q heads) and kcodes/kscales/v8/vscale/kmean (kv heads)."""
    TQ = (offs[2] - offs[1]) // (Hq * 16384)
    TK = (offs[4] - offs[3]) // (Hkv * 16384)
    qc = region(ws_np, offs, 1).view(np.int8).reshape(Hq, TQ, 16384)
    qs = region(ws_np, offs, 2)[: Hq * TQ * 16].view(np.float32).reshape(Hq, TQ, 4)
    kc = region(ws_np, offs, 3).view(np.int8).reshape(Hkv, TK, 16384)
    ks = region(ws_np, offs, 4)[: Hkv * TK * 16].view(np.float32).reshape(Hkv, TK, 4)
    vc = region(ws_np, offs, 5).view(np.uint8).reshape(Hkv, TK, 16384)
    vs = region(ws_np, offs, 6)[: batch * Hkv * 128 * 4].view(np.float32).reshape(batch, Hkv, 128)
    km = region(ws_np, offs, 7)[: batch * Hkv * 128 * 4].view(np.float32).reshape(batch, Hkv, 128)
    out = {}
    for b in range(batch):
        nq = (lens_q[b] + 127) // 128
        nk = (lens_k[b] + 127) // 128
        for h in range(Hq):
            rows = [unswizzle_tile(qc[h, tile0_q[b] + t].view(np.uint8)).view(np.int8) for t in range(nq)]
            codes = np.concatenate(rows, 0)[: lens_q[b]] if rows else np.zeros((0, 128), np.int8)
            scales = qs[h, tile0_q[b]:tile0_q[b] + nq, :2].reshape(-1)[: (lens_q[b] + 63) // 64]
            out[("q", b, h)] = dict(codes=codes, scales=scales)
        for h in range(Hkv):
            rows = [unswizzle_tile(kc[h, tile0_k[b] + t].view(np.uint8)).view(np.int8) for t in range(nk)]
            codes = np.concatenate(rows, 0)[: lens_k[b]] if rows else np.zeros((0, 128), np.int8)
            scales = ks[h, tile0_k[b]:tile0_k[b] + nk, :2].reshape(-1)[: (lens_k[b] + 63) // 64]
            vt = [unswizzle_tile(vc[h, tile0_k[b] + t]) for t in range(nk)]   # [token, d] tiles
            v8 = np.concatenate(vt, 0)[: lens_k[b]] if vt else np.zeros((0, 128), np.uint8)
            out[("k", b, h)] = dict(codes=codes, scales=scales, v8=v8, vscale=vs[b, h], kmean=km[b, h])
    return out
