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
routing of a few rows somewhere in 40 layers, and such a row's hidden state then follows another expert. The test
therefore records both sides' picks at every layer and asserts top-1 agreement >= 99.7% on the rows whose routing
agreed at every layer (the kernels' numerics), and reports the overall agreement and how many rows diverged in
routing, with a loose floor on the overall agreement."""
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
    def __init__(self, model, dev):
        from vllm_espalier_b200 import experts as G
        self.G, self.m, self.dev = G, model, dev
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

    def proj(self, x, m, keep=True):
        """H(H(x * suh) / sqrt(128) -> fp16 @ W) / sqrt(128) * svh in fp32."""
        xh = self.had(x.float() * m.suh.float()).half().float()
        return self.had(xh @ self.W(m, keep)) * m.svh.float()

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
        self.picks = []
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
        return self.had(xh @ W) * head.svh.float()


def test_full_decoder_top1_agreement(dev):
    import bench as B
    model = B.Decoder(dev)
    ref = _Ref(model, dev)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    agree = total = same_routing = agree_same = 0
    for _ in range(STEPS):
        tokens = torch.randint(0, B.VOCAB, (ROWS,), device=dev, generator=g)
        picks = []
        ours = model.forward(tokens, picks).float()
        want = ref.forward(tokens)
        hit = ours.argmax(1) == want.argmax(1)
        routed_alike = torch.ones(ROWS, dtype=torch.bool, device=dev)
        for a, b in zip(picks, ref.picks):
            routed_alike &= (a.long() == b.long()).all(1)
        agree += int(hit.sum())
        total += ROWS
        same_routing += int(routed_alike.sum())
        agree_same += int((hit & routed_alike).sum())
    frac = agree / total
    frac_same = agree_same / max(1, same_routing)
    print(f"top-1 agreement {agree}/{total} = {frac:.4f}; rows routed alike at all {len(model.blocks)} layers: "
          f"{same_routing}/{total}, their top-1 agreement {agree_same}/{same_routing} = {frac_same:.4f}")
    assert same_routing >= total // 2, f"only {same_routing}/{total} rows routed alike"
    assert frac_same >= 0.997, f"top-1 agreement on rows routed alike {agree_same}/{same_routing} = {frac_same:.4f}"
    assert frac >= 0.9, f"overall top-1 agreement {agree}/{total} = {frac:.4f}"
