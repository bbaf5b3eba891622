"""Generate the golden vectors under tests/golden/ (run in the build container).

Source of truth: the reference's committed numerical fixtures
(test/fixtures/numerical/{min_gru,delta_net,mamba,gqa}_random.safetensors, made
by scripts/generate_random_weight_fixtures.py with torch seeds 42/123) and the
reference's own PyTorch model classes in that generator script, imported from
the reference tree (read-only; its main() is not run, nothing is written there).

For each fixture this script loads the weights into the reference's model
class, replays the forward pass with the model's own submodules while
capturing the inputs and outputs of the sequence-mixing op, and asserts that
the replayed model output equals the fixture's ``expected_output`` (and, for
DeltaNet, that the input gradient equals ``gradient.input``).  The captured
op-level vectors are what the oracle is pinned against:

  mingru_fixture.npz     z, c, h per layer; gz, gc = autograd of the
                         reference loop under a seeded N(0,1) upstream dY
  delta_net_fixture.npz  q, k(normalised), v, beta(per element), o per layer;
                         gq, gk, gv, gbeta = autograd under seeded dO
  mamba_fixture.npz      x, dt(clamped), B, C, y per layer (model semantics:
                         fixed A = -(1..N), channel-mean dt in B_bar)
  gqa_fixture.npz        q [B,Hq,L,d], k, v [B,Hkv,L,d], o (causal) per layer;
                         dq, dk, dv = autograd under seeded dO

Usage:  python tests/golden/make_golden.py --reference <reference checkout>
"""
import argparse
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def _load(ref_root, name):
    from safetensors.torch import load_file
    return load_file(os.path.join(ref_root, "test", "fixtures", "numerical",
                                  "%s_random.safetensors" % name))


def _weights(fx):
    return {k[len("weight."):]: v for k, v in fx.items() if k.startswith("weight.")}


def _check(name, got, want, atol):
    err = (got - want).abs().max().item()
    if err > atol:
        raise SystemExit("%s: replay differs from the fixture by %.3g (> %g)" % (name, err, atol))
    print("  %s: replay matches fixture (max abs diff %.2e)" % (name, err))
    return err


def _upstream(t, seed):
    """Seeded N(0,1) upstream gradient for op-level autograd vectors (a plain
    sum() of the model output passes through LayerNorm and leaves the op
    gradients ~1e-15, which would pin nothing)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(t.shape, generator=g)


def _delta_op(q, k, v, beta):
    """The reference generator's sequential delta rule (DeltaNetLayer.forward)."""
    B, L, nh, hd = q.shape
    S = torch.zeros(B, nh, hd, hd, dtype=q.dtype)
    outs = []
    for t in range(L):
        r = torch.einsum("bhij,bhj->bhi", S, k[:, t])
        S = S + torch.einsum("bhi,bhj->bhij", beta[:, t] * (v[:, t] - r), k[:, t])
        outs.append(torch.einsum("bhij,bhj->bhi", S, q[:, t]))
    return torch.stack(outs, dim=1)


def _gqa_op(q, k, v):
    """The reference generator's GQA attention core (GQAAttention.forward)."""
    B, nh, L, hd = q.shape
    g = nh // k.shape[1]
    kr = k.unsqueeze(2).expand(-1, -1, g, -1, -1).reshape(B, nh, L, hd)
    vr = v.unsqueeze(2).expand(-1, -1, g, -1, -1).reshape(B, nh, L, hd)
    scores = torch.matmul(q, kr.transpose(-2, -1)) / (hd ** 0.5)
    mask = torch.triu(torch.ones(L, L), diagonal=1).bool()
    scores = scores.masked_fill(mask, -1e9)
    return torch.matmul(F.softmax(scores, dim=-1), vr)


def make_mingru(gen, ref_root):
    fx = _load(ref_root, "min_gru")
    torch.manual_seed(0)
    model = gen.MinGRUModel(embed_dim=32, hidden_size=64, num_layers=2)
    model.load_state_dict(_weights(fx))
    model.eval()
    x = fx["input.state_sequence"].clone()
    caps = []
    h = model.input_projection(x)
    for layer in model.layers:
        normed = layer.norm(h)
        z = torch.sigmoid(layer.gate(normed))
        c = layer.candidate(normed)
        z.retain_grad(); c.retain_grad()
        B, L, H = z.shape
        st = torch.zeros(B, H)
        outs = []
        for t in range(L):
            st = (1 - z[:, t]) * st + z[:, t] * c[:, t]
            outs.append(st)
        hs = torch.stack(outs, dim=1)
        hs.retain_grad()
        caps.append((z, c, hs))
        h = hs + h
    out = model.final_norm(h)[:, -1]
    err = _check("min_gru", out.detach(), fx["expected_output"], 1e-5)
    d = {"model_replay_err": np.float64(err)}
    for i, (z, c, hs) in enumerate(caps):
        z, c = z.detach().clone().requires_grad_(True), c.detach().clone().requires_grad_(True)
        B, L, H = z.shape
        st = torch.zeros(B, H)
        outs = []
        for t in range(L):
            st = (1 - z[:, t]) * st + z[:, t] * c[:, t]
            outs.append(st)
        hs = torch.stack(outs, dim=1)
        dy = _upstream(hs, 100 + i)
        hs.backward(dy)
        d["z%d" % i] = z.detach().numpy()
        d["c%d" % i] = c.detach().numpy()
        d["h%d" % i] = hs.detach().numpy()
        d["dy%d" % i] = dy.numpy()
        d["gz%d" % i] = z.grad.numpy()
        d["gc%d" % i] = c.grad.numpy()
    np.savez(os.path.join(HERE, "mingru_fixture.npz"), **d)


def make_delta_net(gen, ref_root):
    fx = _load(ref_root, "delta_net")
    model = gen.DeltaNetModel(embed_dim=32, hidden_size=32, num_heads=4, num_layers=2)
    model.load_state_dict(_weights(fx))
    x = fx["input.state_sequence"].clone().requires_grad_(True)
    caps = []
    h = x
    for layer in model.layers:
        normed = layer.norm(h)
        proj = layer.qkvb_proj(normed)
        Hs = layer.hidden_size
        q, k, v, bp = proj[..., :Hs], proj[..., Hs:2 * Hs], proj[..., 2 * Hs:3 * Hs], proj[..., 3 * Hs:]
        B, L = h.shape[:2]
        nh, hd = layer.num_heads, layer.head_dim
        beta = torch.sigmoid(bp).reshape(B, L, nh, hd)
        q = q.reshape(B, L, nh, hd)
        k = F.normalize(k.reshape(B, L, nh, hd), dim=-1, eps=1e-6)
        v = v.reshape(B, L, nh, hd)
        for t_ in (q, k, v, beta):
            t_.retain_grad()
        S = torch.zeros(B, nh, hd, hd)
        outs = []
        for t in range(L):
            r = torch.einsum("bhij,bhj->bhi", S, k[:, t])
            S = S + torch.einsum("bhi,bhj->bhij", beta[:, t] * (v[:, t] - r), k[:, t])
            outs.append(torch.einsum("bhij,bhj->bhi", S, q[:, t]))
        o = torch.stack(outs, dim=1)
        o.retain_grad()
        caps.append((q, k, v, beta, o))
        h = h + layer.out_proj(o.reshape(B, L, nh * hd))
    out = model.final_norm(h)[:, -1]
    err = _check("delta_net", out.detach(), fx["expected_output"], 1e-5)
    out.sum().backward()
    gerr = _check("delta_net gradient.input", x.grad, fx["gradient.input"], 1e-5)
    d = {"model_replay_err": np.float64(err), "grad_replay_err": np.float64(gerr)}
    for i, (q, k, v, beta, o) in enumerate(caps):
        leaves = [t_.detach().clone().requires_grad_(True) for t_ in (q, k, v, beta)]
        o2 = _delta_op(*leaves)
        assert torch.equal(o2.detach(), o.detach())
        do = _upstream(o2, 200 + i)
        o2.backward(do)
        for nm, t_ in zip(("q", "k", "v", "beta"), leaves):
            d["%s%d" % (nm, i)] = t_.detach().numpy()
        d["o%d" % i] = o2.detach().numpy()
        d["do%d" % i] = do.numpy()
        for nm, t_ in zip(("gq", "gk", "gv", "gbeta"), leaves):
            d["%s%d" % (nm, i)] = t_.grad.numpy()
    np.savez(os.path.join(HERE, "delta_net_fixture.npz"), **d)


def make_mamba(gen, ref_root):
    fx = _load(ref_root, "mamba")
    model = gen.MambaModel(embed_dim=32, hidden_size=32, state_size=8, num_layers=2,
                           expand_factor=2, conv_size=4)
    model.load_state_dict(_weights(fx))
    model.eval()
    x = fx["input.state_sequence"].clone()
    caps = []
    orig = gen.MambaBlock._selective_scan

    def capture(self, xa, dt, Bm, Cm):
        y = orig(self, xa, dt, Bm, Cm)
        caps.append((xa.detach(), dt.detach(), Bm.detach(), Cm.detach(), y.detach()))
        return y

    gen.MambaBlock._selective_scan = capture
    try:
        with torch.no_grad():
            out = model(x)
    finally:
        gen.MambaBlock._selective_scan = orig
    err = _check("mamba", out, fx["expected_output"], 1e-5)
    d = {"model_replay_err": np.float64(err)}
    for i, (xa, dt, Bm, Cm, y) in enumerate(caps):
        d["x%d" % i], d["dt%d" % i], d["B%d" % i], d["C%d" % i], d["y%d" % i] = (
            xa.numpy(), dt.numpy(), Bm.numpy(), Cm.numpy(), y.numpy())
    np.savez(os.path.join(HERE, "mamba_fixture.npz"), **d)


def make_gqa(gen, ref_root):
    fx = _load(ref_root, "gqa")
    model = gen.GQAModel(embed_dim=32, hidden_size=32, num_heads=4, num_kv_heads=2, num_layers=2)
    model.load_state_dict(_weights(fx))
    model.eval()
    x = fx["input.state_sequence"].clone()
    caps = []
    h = x
    for blk in model.blocks:
        att = blk.attn
        a_in = blk.attn_norm(h)
        B, L, _ = a_in.shape
        hd, nh, nkv = att.head_dim, att.num_heads, att.num_kv_heads
        q = att.q_proj(a_in).reshape(B, L, nh, hd).transpose(1, 2).contiguous()
        k = att.k_proj(a_in).reshape(B, L, nkv, hd).transpose(1, 2).contiguous()
        v = att.v_proj(a_in).reshape(B, L, nkv, hd).transpose(1, 2).contiguous()
        for t_ in (q, k, v):
            t_.retain_grad()
        g = nh // nkv
        kr = k.unsqueeze(2).expand(-1, -1, g, -1, -1).reshape(B, nh, L, hd)
        vr = v.unsqueeze(2).expand(-1, -1, g, -1, -1).reshape(B, nh, L, hd)
        scores = torch.matmul(q, kr.transpose(-2, -1)) / (hd ** 0.5)
        mask = torch.triu(torch.ones(L, L), diagonal=1).bool()
        scores = scores.masked_fill(mask, -1e9)
        o = torch.matmul(F.softmax(scores, dim=-1), vr)
        o.retain_grad()
        caps.append((q, k, v, o))
        h = h + att.out_proj(o.transpose(1, 2).reshape(B, L, nh * hd))
        f = blk.ffn_down(F.gelu(blk.ffn_up(blk.ffn_norm(h))))
        h = h + f
    out = model.final_norm(h)[:, -1]
    err = _check("gqa", out.detach(), fx["expected_output"], 1e-5)
    d = {"model_replay_err": np.float64(err)}
    for i, (q, k, v, o) in enumerate(caps):
        leaves = [t_.detach().clone().requires_grad_(True) for t_ in (q, k, v)]
        o2 = _gqa_op(*leaves)
        assert torch.allclose(o2.detach(), o.detach(), atol=1e-6)
        do = _upstream(o2, 300 + i)
        o2.backward(do)
        for nm, t_ in zip(("q", "k", "v"), leaves):
            d["%s%d" % (nm, i)] = t_.detach().numpy()
        d["o%d" % i] = o2.detach().numpy()
        d["do%d" % i] = do.numpy()
        d["dq%d" % i], d["dk%d" % i], d["dv%d" % i] = (t_.grad.numpy() for t_ in leaves)
    np.savez(os.path.join(HERE, "gqa_fixture.npz"), **d)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("EDIFICE_REFERENCE_ROOT"),
                    help="the reference checkout (default: $EDIFICE_REFERENCE_ROOT)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or EDIFICE_REFERENCE_ROOT")
    sys.path.insert(0, os.path.join(args.reference, "scripts"))
    import generate_random_weight_fixtures as gen  # the reference's own model classes
    torch.set_grad_enabled(True)
    make_mingru(gen, args.reference)
    make_delta_net(gen, args.reference)
    make_mamba(gen, args.reference)
    make_gqa(gen, args.reference)
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
