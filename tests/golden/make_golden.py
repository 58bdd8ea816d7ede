"""Generate the golden fixtures in this folder from the reference's own kernels.

Runs the reference's ``solution/kernels`` modules (RMSNorm, SwiGLU, RoPE and the
chunked cross-entropy) on the CPU through Triton's interpreter
(``TRITON_INTERPRET=1``) on small seeded inputs, and stores inputs and outputs as
``*.pt`` files next to this script. The fixtures pin the CPU oracle
(``tests/test_oracle_golden.py``) and the CUDA kernels (``tests/test_gpu_golden.py``).

Usage (needs the reference checkout; the fixtures themselves are committed)::

    python tests/golden/make_golden.py --reference /path/to/Auspex_Soup_Demo
"""

from __future__ import annotations

import argparse
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="checkout of the reference project (its solution/ package is imported)")
    args = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    # Triton's cache goes to a throwaway folder; nothing in it is read.
    os.environ.setdefault("TRITON_CACHE_DIR", tempfile.mkdtemp(prefix="golden_triton_"))
    sys.path.insert(0, args.reference)

    import torch
    from solution.kernels import chunked_ce, rmsnorm, rope, swiglu

    def save(name, obj):
        path = os.path.join(HERE, name)
        torch.save(obj, path)
        print(f"wrote {path} ({os.path.getsize(path)} B)")

    # ---------------- RMSNorm: forward + backward (dx, dw) -----------------
    cases = []
    for tag, shape, dtype in [("f32_d96", (2, 8, 96), torch.float32),
                              ("f32_d1536", (16, 1536), torch.float32),
                              ("bf16_d1536", (4, 5, 1536), torch.bfloat16)]:
        g = torch.Generator().manual_seed(100 + len(cases))
        D = shape[-1]
        x = torch.randn(shape, generator=g).to(dtype)
        w = (1.0 + 0.1 * torch.randn(D, generator=g)).to(dtype)
        dy = torch.randn(shape, generator=g).to(dtype)
        xr = x.clone().requires_grad_(True)
        wr = w.clone().requires_grad_(True)
        y = rmsnorm.fast_rms_norm(xr, wr, 1e-6)
        y.backward(dy)
        cases.append(dict(tag=tag, x=x, w=w, dy=dy, eps=1e-6, y=y.detach(),
                          dx=xr.grad.detach(), dw=wr.grad.detach()))
    save("rmsnorm.pt", cases)

    # ---------------- SwiGLU: forward + backward ---------------------------
    cases = []
    for tag, shape, dtype in [("bf16_ragged", (3, 7, 1000), torch.bfloat16),
                              ("f32_wide", (2, 2144), torch.float32),
                              ("bf16_big", (4, 8960), torch.bfloat16)]:
        g = torch.Generator().manual_seed(200 + len(cases))
        gate = torch.randn(shape, generator=g).to(dtype)
        up = torch.randn(shape, generator=g).to(dtype)
        dy = torch.randn(shape, generator=g).to(dtype)
        gr = gate.clone().requires_grad_(True)
        ur = up.clone().requires_grad_(True)
        out = swiglu.fast_swiglu(gr, ur)
        out.backward(dy)
        cases.append(dict(tag=tag, gate=gate, up=up, dy=dy, out=out.detach(),
                          dgate=gr.grad.detach(), dup=ur.grad.detach()))
    save("swiglu.pt", cases)

    # ---------------- RoPE: forward + backward -----------------------------
    def hf_cos_sin(B, S, D, theta, dtype):
        inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))
        pos = torch.arange(S)[None, :].expand(B, -1).float()
        freqs = (inv[None, :, None].expand(B, -1, 1) @ pos[:, None, :]).transpose(1, 2)
        emb = torch.cat((freqs, freqs), dim=-1)
        return emb.cos().to(dtype), emb.sin().to(dtype)  # [B, S, D]

    cases = []
    # HF layout: [B,S,H,D] projections viewed as [B,H,S,D] (strided), cos/sin [B,1,S,D].
    g = torch.Generator().manual_seed(300)
    B, S, H, HK, D = 2, 16, 12, 2, 128
    q = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16).transpose(1, 2)
    k = torch.randn(B, S, HK, D, generator=g).to(torch.bfloat16).transpose(1, 2)
    dq = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
    dk = torch.randn(B, HK, S, D, generator=g).to(torch.bfloat16)
    cos, sin = hf_cos_sin(B, S, D, 1e6, torch.bfloat16)
    for tag, x, dy in [("bf16_q_strided", q, dq), ("bf16_k_strided", k, dk)]:
        xr = x.detach().clone().requires_grad_(True)  # clone keeps the strides
        out = rope.apply_fast_rope(xr, cos.unsqueeze(1), sin.unsqueeze(1))
        out.backward(dy)
        cases.append(dict(tag=tag, x=x, dy=dy, cos=cos.unsqueeze(1), sin=sin.unsqueeze(1),
                          out=out.detach(), dx=xr.grad.detach()))
    g = torch.Generator().manual_seed(301)
    x = torch.randn(1, 3, 9, 128, generator=g)
    dy = torch.randn(1, 3, 9, 128, generator=g)
    c1, s1 = hf_cos_sin(1, 9, 128, 10000.0, torch.float32)
    xr = x.clone().requires_grad_(True)
    out = rope.apply_fast_rope(xr, c1[:, None], s1[:, None])
    out.backward(dy)
    cases.append(dict(tag="f32_contig", x=x, dy=dy, cos=c1[:, None], sin=s1[:, None],
                      out=out.detach(), dx=xr.grad.detach()))
    save("rope.pt", cases)

    # ---------------- CE kernel on a logits buffer (in place) --------------
    cases = []
    for tag, N, V, dtype in [("f16_v1000", 8, 1000, torch.float16),
                             ("bf16_v4099_two_tiles", 5, 4099, torch.bfloat16),
                             ("f16_v4096", 4, 4096, torch.float16)]:
        g = torch.Generator().manual_seed(400 + len(cases))
        logits = torch.randn(N, V, generator=g).to(dtype)
        targets = torch.randint(0, V, (N,), generator=g)
        targets[0] = -100
        # exact ties of the row maximum pin first-index argmax semantics
        logits[1, 10] = 9.0
        logits[1, V - 7] = 9.0
        targets[1] = 10 if N % 2 == 0 else V - 7
        if V > 4096:
            logits[2, 100] = 9.5
            logits[2, 4097] = 9.5
            targets[2] = 4097
        den = float((targets != -100).sum().item())
        buf = logits.clone()
        losses = torch.empty(N, dtype=torch.float32)
        ents = torch.empty(N, dtype=torch.float32)
        corr = torch.empty(N, dtype=torch.int32)
        chunked_ce._chunked_cross_entropy_fused_kernel[(N,)](
            buf, targets, losses, ents, corr, stride_logits_row=buf.stride(0), V=V,
            denominator=den, ignore_index=-100, BLOCK_V=4096, num_warps=8, num_stages=2)
        cases.append(dict(tag=tag, logits=logits, targets=targets, denominator=den,
                          losses=losses, entropies=ents, correct=corr, grad=buf))
    save("ce_kernel.pt", cases)

    # ---------------- Chunked head loss (autograd Function) ----------------
    Fn = chunked_ce.make_triton_chunked_loss_function()
    cases = []
    for tag, B, S, D, V, chunk, dtype in [("f32_ragged_chunk", 2, 40, 64, 1000, 16, torch.float32),
                                          ("bf16_s64", 2, 64, 96, 4099, 32, torch.bfloat16)]:
        g = torch.Generator().manual_seed(500 + len(cases))
        hidden = torch.randn(B, S, D, generator=g).to(dtype)
        W = (0.02 * torch.randn(V, D, generator=g)).to(dtype) * 8.0
        target = torch.randint(0, V, (B, S), generator=g)
        drop = torch.rand(B, S, generator=g) < 0.1
        target[drop] = -100
        den = float((target != -100).sum().item())
        head = torch.nn.Linear(D, V, bias=False, dtype=dtype)
        with torch.no_grad():
            head.weight.copy_(W)
        h = hidden.clone().requires_grad_(True)
        loss, ent, tok, corr = Fn.apply(h, head, target, chunk, den, -100, True)
        loss.backward()
        cases.append(dict(tag=tag, hidden=hidden, weight=W, target=target, chunk=chunk,
                          denominator=den, loss=loss.detach(), entropy=ent, token_loss=tok,
                          correct=corr, dhidden=h.grad.detach()))
    save("chunked_loss.pt", cases)


if __name__ == "__main__":
    main()
