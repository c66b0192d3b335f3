"""Host emulation of the resident kernel's data movement -- test infrastructure.

Replays, with numpy, exactly the index arithmetic of
low_latency_inference_gpu_b200/csrc/resident_kernel.cuh on the plan and the
packed per-CTA shared-memory images returned by ``ll_plan_net``: stage input
staging, every layer mode's dot products and epilogue, the DSMEM pushes into
peers' buffers, the inter-cluster handoff and the rank-0 gather.  Every
shared-memory access is bounds-checked against the buffer it must stay in, so a
plan or packing bug shows up here on the CPU, never as a GPU fault.
"""
from __future__ import annotations

import numpy as np

import low_latency_inference_gpu_b200 as ll

BUF_X, BUF_A, BUF_B, BUF_L, BUF_G, BUF_STAGE = range(6)
LM_REPLICATED, LM_ALLGATHER, LM_LOCAL, LM_KSPLIT, LM_RGATHER, LM_GLOBAL = range(6)
UNIT = {ll.W_F32: 4, ll.W_BF16: 8, ll.W_I8: 16}
WB = {ll.W_F32: 4, ll.W_BF16: 2, ll.W_I8: 1}


def _bf16(v):
    v = np.asarray(v, np.float32)
    u = v.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return (u.astype(np.uint32) << 16).view(np.float32)


def _act(v, act):
    if act == ll.ACT_RELU:
        return np.maximum(v, np.float32(0))
    if act == ll.ACT_GELU:
        from math import erf
        return np.array([0.5 * x * (1.0 + erf(x / np.sqrt(2.0))) for x in v.ravel()], np.float32).reshape(v.shape)
    return v


class Smem:
    """One CTA's shared memory: image bytes + float buffers, with region checks."""

    def __init__(self, plan, image: np.ndarray):
        self.plan = plan
        self.size = plan.smem_bytes
        self.bytes = np.zeros(self.size, np.uint8)
        assert image.size <= plan.buf_off[BUF_X], "image overlaps the buffers"
        self.bytes[: image.size] = image
        ends = list(plan.buf_off[1:6]) + [plan.smem_bytes]
        self.region = {i: (plan.buf_off[i], ends[i]) for i in range(6)}

    def fview(self, buf):
        lo, hi = self.region[buf]
        return self.bytes[lo:hi].view(np.float32)

    def check(self, buf, idx):
        lo, hi = self.region[buf]
        n = (hi - lo) // 4
        idx = np.asarray(idx)
        assert idx.min() >= 0 and idx.max() < n, f"buffer {buf}: index {idx.min()}..{idx.max()} outside [0,{n})"

    def read(self, buf, idx):
        self.check(buf, idx)
        return self.fview(buf)[idx]

    def write(self, buf, idx, vals):
        self.check(buf, idx)
        self.fview(buf)[idx] = vals

    def weights(self, L, stage_img_bytes):
        nbytes = L.R * L.K * WB[L.wtype]
        assert L.w_off + nbytes <= stage_img_bytes, "weight slice outside the image"
        raw = self.bytes[L.w_off: L.w_off + nbytes]
        if L.wtype == ll.W_F32:
            w = raw.view(np.float32)
        elif L.wtype == ll.W_BF16:
            w = (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            w = raw.view(np.int8).astype(np.float32)
        return w.reshape(L.R, L.K)

    def vec(self, off, n, stage_img_bytes):
        assert off + 4 * n <= stage_img_bytes
        return self.bytes[off: off + 4 * n].view(np.float32)


def run(plan, images: np.ndarray, x: np.ndarray, out_dim: int) -> np.ndarray:
    """Emulate one request of n_rows = x.shape[0] through the planned kernel; returns y."""
    S, C = plan.n_stages, plan.cluster_size
    nrows, in_dim = x.shape
    assert nrows <= plan.bmax4
    ctas = [[Smem(plan, images[(s * C + r) * plan.image_stride:(s * C + r) * plan.image_stride
                               + plan.image_bytes[s]]) for r in range(C)] for s in range(S)]
    xfer = {}
    y = None
    for s in range(S):
        img_bytes = plan.image_bytes[s]
        ld = plan.stage_in_ld[s]
        # ---- stage input ----
        for r in range(C):
            sm = ctas[s][r]
            for b in range(nrows):
                if s == 0:
                    v = x[b].astype(np.float32)
                    if plan.act_bf16:
                        v = _bf16(v)
                    sm.write(BUF_X, b * ld + np.arange(in_dim), v)
                else:
                    src = xfer[s - 1]
                    sm.write(BUF_X, b * ld + np.arange(ld), src[b * ld:(b + 1) * ld])
        # ---- layers ----
        for l in range(plan.stage_first[s], plan.stage_last[s] + 1):
            L = plan.layers[l]
            pushes = []  # (dst_rank, buf, idx, vals)
            for r in range(C):
                sm = ctas[s][r]
                W = sm.weights(L, img_bytes)
                assert L.K % UNIT[L.wtype] == 0
                bias = sm.vec(L.b_off, L.R, img_bytes)
                scale = sm.vec(L.s_off, L.R, img_bytes) if L.s_off != 0xFFFFFFFF else None
                inp = np.stack([sm.read(L.in_buf, b * L.in_ld + np.arange(L.K)) for b in range(nrows)])
                acc = (inp.astype(np.float64) @ W.T.astype(np.float64)).astype(np.float32)  # [nrows, R]
                if L.mode == LM_KSPLIT:
                    stg = acc
                else:
                    v = acc * scale[None, :] if scale is not None else acc
                    v = _act(v + bias[None, :], L.act)
                    if L.round_out and L.mode != LM_RGATHER:
                        v = _bf16(v)
                    stg = v.astype(np.float32)
                if L.mode in (LM_REPLICATED, LM_LOCAL):
                    for b in range(nrows):
                        sm.write(L.out_buf, b * L.out_ld + np.arange(L.R), stg[b])
                    continue
                for b in range(nrows):
                    sm.write(BUF_STAGE, b * L.R + np.arange(L.R), stg[b])
                if L.mode == LM_ALLGATHER:
                    for d in range(C):
                        for b in range(nrows):
                            pushes.append((d, L.out_buf, b * L.out_ld + r * L.R + np.arange(L.R), stg[b]))
                elif L.mode == LM_KSPLIT:
                    base = r * plan.bmax4 * L.R
                    for b in range(nrows):
                        pushes.append((0, BUF_G, base + b * L.R + np.arange(L.R), stg[b]))
                elif L.mode == LM_RGATHER:
                    for b in range(nrows):
                        pushes.append((0, BUF_G, b * L.Mp + r * L.R + np.arange(L.R), stg[b]))
                elif L.mode == LM_GLOBAL:
                    buf = xfer.setdefault(s, np.zeros(plan.bmax4 * L.Mp, np.float32))
                    for b in range(nrows):
                        idx = b * L.Mp + r * L.R + np.arange(L.R)
                        assert idx.max() < buf.size
                        buf[idx] = stg[b]
            for d, buf, idx, vals in pushes:
                ctas[s][d].write(buf, idx, vals)
        # ---- final writer ----
        if s == S - 1:
            Lf = plan.layers[plan.n_layers - 1]
            sm = ctas[s][0]
            y = np.zeros((nrows, out_dim), np.float32)
            fb = sm.vec(Lf.b_off, Lf.R, img_bytes)
            fs = sm.vec(Lf.s_off, Lf.R, img_bytes) if Lf.s_off != 0xFFFFFFFF else None
            for b in range(nrows):
                for o in range(out_dim):
                    if Lf.mode == LM_KSPLIT:
                        acc = np.float32(0)
                        for c in range(C):
                            acc = np.float32(acc + sm.read(BUF_G, (c * plan.bmax4 + b) * Lf.R + o))
                        if fs is not None:
                            acc = np.float32(acc * fs[o])
                        y[b, o] = _act(np.array([acc + fb[o]], np.float32), Lf.act)[0]
                    else:
                        y[b, o] = sm.read(BUF_G, b * Lf.Mp + o)
    return y
