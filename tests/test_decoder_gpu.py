"""BASELINE configs[4] parity: top-1 agreement between the full synthetic decoder through this library and the
reference's decode-then-matmul composition (vllm_espalier/ops.py:45-51 for every projection, experts.py routed2
arithmetic for the experts) in fp32 torch on the same GPU, over decoded weights that are bit-identical to the
reference's decode.

Both sides share the model (bench.Decoder: 40 layers, config-2 projections, config-3 MoE, 6-bit mcg LM head), the
embedding, the RMSNorms, the residual adds and the stand-in mixer cores; they differ in everything on this path:
  ours       fused dense kernels, fused routing, grouped expert kernels (fp16 activations x decoded weights on the
             tensor cores, fp32 sums in this library's orders);
  reference  dequant -> fp32 matmul per matrix, exact routing (the CPU oracle's fp64 logits rounded once to bf16,
             lowest id on ties), per-expert fp32 gate/up/SwiGLU/down, slot-ordered fp32 combine.
Rows are teacher-forced (the same random tokens on both sides at every step).

With random weights the router's top-8 boundary is dense with near-ties (the 8th and 9th of 256 N(0, 1) logits lie
~0.06 apart against a bf16 resolution of 0.016 there), so last-ulp differences between two correct paths flip the
routing of rows somewhere in 40 layers, and such a row's hidden state then follows another expert. BASELINE's 99.7%
presumes a trained model's margins. The test therefore measures the floor any implementation faces: the same
reference composition run a second time with another legitimate fp32 summation order (each projection's K split in
two halves) and compared with the first. It asserts that this library agrees with the reference at least as well as
that second reference run does (within 3 points), and prints both agreements and both runs' per-layer routing
agreement with the reference. (For int5 / int6 this library sums q * x over the exact grid index q and applies the
codebook step c to the fp32 sum, as the reference's fused dense kernel does with its codebooks 22 / 23; the
decode-then-matmul path multiplies by the fp16-rounded q * c, a relative difference of at most 2^-11 a weight, which
already moves a few percent of the first layer's near-tied routing boundaries.)"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

STEPS, ROWS = 8, 32


def _hadamard(dev):
    h = torch.ones(1, 1, dtype=torch.float64)
    while h.shape[0] < 128:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return (h / np.sqrt(128.0)).to(torch.float32).to(dev)


class _Ref:
    def __init__(self, model, dev, split_k: bool = False):
        from vllm_espalier_b200 import experts as G
        self.G, self.m, self.dev, self.split_k = G, model, dev, split_k
        self.H = _hadamard(dev)
        self.cache = {}

    def had(self, v):
        return (v.reshape(*v.shape[:-1], -1, 128) @ self.H).reshape(v.shape)

    def W(self, m, keep=True):
        key = id(m)
        if key in self.cache:
            return self.cache[key]
        w = self.G.dequant(m.trellis, m.K, m.cb).float()
        if keep:
            self.cache[key] = w
        return w

    def mm(self, xh, W):
        if not self.split_k:
            return xh @ W
        h = W.shape[0] // 2
        return xh[:, :h] @ W[:h] + xh[:, h:] @ W[h:]

    def proj(self, x, m, keep=True):
        """H(H(x * suh) / sqrt(128) -> fp16 @ W) / sqrt(128) * svh in fp32."""
        xh = self.had(x.float() * m.suh.float()).half().float()
        return self.had(self.mm(xh, self.W(m, keep))) * m.svh.float()

    def dense(self, x, d):
        return torch.cat([self.proj(x, m) for m in d.mats], 1).to(torch.bfloat16)

    def moe(self, h, layer):
        L, gate, ex, sh = layer
        R = h.shape[0]
        hb = h.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        gb = gate.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        sgb = L.gate_w.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        k = 8
        pick, wts, _ = O.route(hb, gb, k, sgb, L.shared_id)
        self.picks.append(torch.from_numpy(pick).to(self.dev))
        self.routes.append((torch.from_numpy(np.ascontiguousarray(pick[:, :k])).to(self.dev),
                            torch.from_numpy(np.ascontiguousarray(wts[:, :k])).to(self.dev)))
        ys = {}
        for e in np.unique(pick):
            rows, slots = np.nonzero(pick == e)
            mats = sh if e == L.shared_id else ex[e]
            x = h[torch.from_numpy(rows).to(self.dev)]
            gg, uu = self.proj(x, mats[0], keep=False), self.proj(x, mats[1], keep=False)
            act = gg / (1 + torch.exp(-gg)) * uu            # silu(gate) * up, fp32 (act_mode 1)
            y = self.proj(act, mats[2], keep=False)
            for i, (r, j) in enumerate(zip(rows, slots)):
                ys[(int(r), int(j))] = y[i]
        out = torch.zeros(R, h.shape[1], device=self.dev)
        out_sh = torch.zeros(R, h.shape[1], device=self.dev)
        w = torch.from_numpy(wts).to(self.dev)
        for r in range(R):
            for j in range(k):
                out[r] = out[r] + w[r, j] * ys[(r, j)]
            out_sh[r] = w[r, k] * ys[(r, k)]
        return out.to(torch.bfloat16), out_sh.to(torch.bfloat16)

    def forward(self, tokens):
        import bench as B
        m = self.m
        self.picks, self.routes = [], []
        x = m.embed[tokens]
        for blk, layer in zip(m.blocks, m.moe):
            h = B.rmsnorm(x, blk["n1"])
            core = B.mixer_core(self.dense(h, blk["qkv"]), blk["attention"])
            x = B.residual(x, self.dense(core, blk["o"]))
            h = B.rmsnorm(x, blk["n2"])
            out, sh = self.moe(h, layer)
            x = B.residual(x, out, sh)
        hf = B.rmsnorm(x, m.final)
        head = m.head.mats[0]
        W = self.W(head, keep=False)
        xh = self.had(hf.float() * head.suh.float()).half().float()
        return self.had(self.mm(xh, W)) * head.svh.float()


def test_full_decoder_top1_agreement(dev):
    import bench as B
    model = B.Decoder(dev)
    ref, alt = _Ref(model, dev), _Ref(model, dev, split_k=True)
    alt.cache = ref.cache                        # the same decoded weights
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    n_layers = len(model.blocks)
    agree = agree_alt = total = 0
    alike, alike_alt = torch.zeros(n_layers), torch.zeros(n_layers)
    for _ in range(STEPS):
        tokens = torch.randint(0, B.VOCAB, (ROWS,), device=dev, generator=g)
        picks = []
        ours = model.forward(tokens, picks).float()
        want = ref.forward(tokens)
        other = alt.forward(tokens)
        agree += int((ours.argmax(1) == want.argmax(1)).sum())
        agree_alt += int((other.argmax(1) == want.argmax(1)).sum())
        total += ROWS
        for i, (a, b, c) in enumerate(zip(picks, ref.picks, alt.picks)):
            alike[i] += float((a.long() == b.long()).all(1).float().sum())
            alike_alt[i] += float((c.long() == b.long()).all(1).float().sum())
    alike /= total
    alike_alt /= total
    frac, frac_alt = agree / total, agree_alt / total
    print(f"top-1 agreement with the reference: this library {agree}/{total} = {frac:.4f}; the reference with "
          f"another fp32 order {agree_alt}/{total} = {frac_alt:.4f}; rows routed alike by layer (this library / other "
          f"order): first {alike[0]:.3f} / {alike_alt[0]:.3f}, mean {alike.mean():.3f} / {alike_alt.mean():.3f}")
    assert frac >= frac_alt - 0.03, f"top-1 agreement {frac:.4f} vs the reference's own order floor {frac_alt:.4f}"


FORCED_STEPS = 16          # 512 rows: 99.7% allows one disagreement


def test_forced_routing_top1_agreement(dev):
    """The arithmetic alone: every layer of this library's decoder is fed the reference side's routing (its exact
    picks and renormalised weights, from the CPU oracle on the reference's own hidden state), so no row can follow
    another expert, and the dense, expert and head arithmetic must give the reference's top-1 token on at least 99.7%
    of rows."""
    import bench as B
    model = B.Decoder(dev)
    ref = _Ref(model, dev)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    agree = total = 0
    for _ in range(FORCED_STEPS):
        tokens = torch.randint(0, B.VOCAB, (ROWS,), device=dev, generator=g)
        want = ref.forward(tokens)
        ours = model.forward(tokens, forced=ref.routes).float()
        agree += int((ours.argmax(1) == want.argmax(1)).sum())
        total += ROWS
    frac = agree / total
    print(f"forced-routing top-1 agreement with the reference: {agree}/{total} = {frac:.4f}")
    assert frac >= 0.997, f"top-1 agreement {frac:.4f} with both sides on the same routing"
