"""Generate the golden fixtures in this folder from the reference implementation itself.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py /path/to/muon_sr_checkout

It imports bab2min/muon_sr 0.1.2 with ``TRITON_INTERPRET=1`` so that its Triton kernels
run on CPU tensors, and its ``_newton_schulz`` and optimizer classes on CPU tensors, on
small seeded inputs, and writes the inputs and outputs as ``.npz`` files next to this
script. The reference ships no tests or golden vectors, so these fixtures are what pins
the CPU oracle (``oracle/``) and the CUDA engine to the reference's behaviour. Nothing at
test time reads the reference checkout; only these files.
"""
import os
import random
import sys

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def from_bits(b) -> torch.Tensor:
    return torch.from_numpy(np.asarray(b, dtype=np.uint16).view(np.int16).copy()).view(torch.bfloat16)


def randn_bf16(rng, n, std):
    return torch.from_numpy((rng.standard_normal(n) * std).astype(np.float32)).bfloat16()


def save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrays)
    print("wrote", path, sum(a.nbytes for a in map(np.asarray, arrays.values())), "bytes")


def main(ref_root):
    sys.path.insert(0, ref_root)
    import triton
    import triton.language as tl
    from muon_sr import triton_adamw as ta
    from muon_sr import triton_muon_sr as tm
    from muon_sr import triton_adamw_8bit as t8
    from muon_sr import muon_sr as ms

    rng = np.random.default_rng(20261201)

    # ---- Philox: tl.randint words for the seeds and 32-bit counters the kernels use ----
    @triton.jit
    def _probe(out_ptr, seed, base, n, ADD: tl.constexpr, BLOCK: tl.constexpr):
        offs = base + tl.program_id(0).to(tl.int64) * BLOCK + tl.arange(0, BLOCK)
        r = tl.randint(seed + ADD, offs.to(tl.int32)).to(tl.int32)
        tl.store(out_ptr + tl.arange(0, BLOCK) + tl.program_id(0) * BLOCK, r,
                 mask=tl.program_id(0) * BLOCK + tl.arange(0, BLOCK) < n)

    seeds = np.array([0, 1, 12345, 2**31 - 2, 2**31 - 1, 2**31, 2**32 - 2, 2**32 - 1], np.uint64)
    bases = np.array([0, 2**31 - 16, 2**32 - 16, 5 * 2**32 + 7], np.uint64)
    words = np.zeros((len(seeds), 3, len(bases), 32), np.uint32)
    for i, s in enumerate(seeds.tolist()):
        for add in range(3):
            for j, b in enumerate(bases.tolist()):
                o = torch.zeros(32, dtype=torch.int32)
                _probe[(1,)](o, s, b, 32, ADD=add, BLOCK=32)
                words[i, add, j] = o.numpy().view(np.uint32)
    save("philox.npz", seeds=seeds, bases=bases, words=words)

    # ---- SR gradient accumulation (triton_adamw.py:206-229) ----
    n = 2053
    acc = randn_bf16(rng, n, 1e-3)
    g = randn_bf16(rng, n, 1e-3 / 16)
    outs = []
    gseeds = np.array([987654321, 3000000001], np.uint64)
    for s in gseeds.tolist():
        a = acc.clone()
        ta._grad_accum_kernel[(triton.cdiv(n, 1024),)](a, g, n, s, BLOCK_SIZE=1024)
        outs.append(bits(a))
    save("grad_accum.npz", acc=bits(acc), grad=bits(g), seeds=gseeds, out=np.stack(outs))

    # ---- Muon prepare / apply (triton_muon_sr.py:18-80) ----
    n = 3001
    g = randn_bf16(rng, n, 1e-3)
    buf = randn_bf16(rng, n, 1e-3)
    pseeds = np.array([tm._deterministic_seed(3, 1, 0), tm._deterministic_seed(7, 10002, 0)], np.uint64)
    res = {}
    for nest in (0, 1):
        for k, s in enumerate(pseeds.tolist()):
            b = buf.clone()
            upd = torch.empty(n, dtype=torch.bfloat16)
            tm._muon_prepare_kernel[(triton.cdiv(n, 1024),)](g, b, upd, 0.95, bool(nest), n, s, BLOCK_SIZE=1024)
            res[f"buf_{nest}_{k}"] = bits(b)
            res[f"upd_{nest}_{k}"] = bits(upd)
    save("muon_prepare.npz", grad=bits(g), buf=bits(buf), seeds=pseeds, beta=np.float64(0.95), **res)

    p = randn_bf16(rng, n, 0.02)
    upd = randn_bf16(rng, n, 0.02)
    aseeds = np.array([tm._deterministic_seed(3, 20001, 1), tm._deterministic_seed(9, 5, 1)], np.uint64)
    cases = [(0.02, 0.01, (96, 32)), (0.05, 0.0, (32, 96))]
    outs = []
    for (lr, wd, shape), s in zip(cases, aseeds.tolist()):
        q = p.clone()
        tm._muon_apply_kernel[(triton.cdiv(n, 1024),)](q, upd, lr, wd, tm._ns_scale(shape), n, s, BLOCK_SIZE=1024)
        outs.append(bits(q))
    save("muon_apply.npz", p=bits(p), upd=bits(upd), seeds=aseeds,
         lr=np.array([c[0] for c in cases]), wd=np.array([c[1] for c in cases]),
         scale=np.array([tm._ns_scale(c[2]) for c in cases]), out=np.stack(outs))

    # ---- AdamW-SR (triton_adamw.py:9-114) ----
    p = randn_bf16(rng, n, 0.02)
    g = randn_bf16(rng, n, 1e-3)
    m = randn_bf16(rng, n, 1e-4)
    v = torch.from_numpy(np.abs(rng.standard_normal(n) * 1e-7).astype(np.float32)).bfloat16()
    cases = [(1, 7), (5, 2**31 - 1), (1000, 2**32 - 1)]
    res = {}
    for k, (step, idx) in enumerate(cases):
        q, mm, vv = p.clone(), m.clone(), v.clone()
        # pass the seed through param_idx so edge seeds are reachable: seed = (step*C1 ^ idx*C2)
        ta._adamw_step(q, g, mm, vv, lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-10,
                       weight_decay=0.01, step=step, param_idx=idx)
        res[f"p_{k}"], res[f"m_{k}"], res[f"v_{k}"] = bits(q), bits(mm), bits(vv)
    # direct kernel launches with edge seeds (2^31-1 wraps seed+1/seed+2 in i32)
    edge = np.array([2**31 - 2, 2**31 - 1, 2**32 - 2], np.uint64)
    for k, s in enumerate(edge.tolist()):
        q, mm, vv = p.clone(), m.clone(), v.clone()
        ta._adamw_kernel[(triton.cdiv(n, 1024),)](q, g, mm, vv, 3e-4, 0.9, 0.95, 1e-10, 0.01,
                                                   1 - 0.9 ** 3, (1 - 0.95 ** 3) ** 0.5, n, s, BLOCK_SIZE=1024)
        res[f"ep_{k}"], res[f"em_{k}"], res[f"ev_{k}"] = bits(q), bits(mm), bits(vv)
    save("adamw.npz", p=bits(p), g=bits(g), m=bits(m), v=bits(v),
         steps=np.array([c[0] for c in cases]), idx=np.array([c[1] for c in cases], np.uint64),
         edge_seeds=edge, **res)

    # ---- 8-bit blockwise AdamW (triton_adamw_8bit.py:14-99) ----
    Q1 = t8.create_dynamic_map(True)
    Q2 = t8.create_dynamic_map(False)
    res = {"qmap1": Q1.numpy(), "qmap2": Q2.numpy()}
    # quantiser on special values: every code point, midpoints, tiny values, signed zero
    xs = np.concatenate([
        Q1.numpy(), ((Q1[1:] + Q1[:-1]) / 2).numpy(), np.nextafter(((Q1[1:] + Q1[:-1]) / 2).numpy(), 2),
        np.nextafter(((Q1[1:] + Q1[:-1]) / 2).numpy(), -2),
        np.array([0.0, -0.0, 1e-9, -1e-9, 2.7e-7, -2.7e-7, 1.0, -1.0], np.float32),
        rng.uniform(-1, 1, 1500).astype(np.float32),
        (rng.standard_normal(500) * 1e-3).astype(np.float32)]).astype(np.float32)
    xu = np.abs(xs)

    # the jitted probe resolves names through this module's globals
    globals()["_ref_quantize"] = t8._quantize

    @triton.jit
    def _qprobe(X, OUT, Q, N, SIGNED: tl.constexpr, BLOCK: tl.constexpr):
        offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
        msk = offs < N
        x = tl.load(X + offs, msk, other=0.)
        tl.store(OUT + offs, _ref_quantize(x, Q, SIGNED), msk)

    for name, x, Q, sgn in (("qs", xs, Q1, True), ("qu", xu, Q2, False)):
        o = torch.zeros(x.size, dtype=torch.uint8)
        _qprobe[(triton.cdiv(x.size, 256),)](torch.from_numpy(x), o, Q, x.size, SIGNED=sgn, BLOCK=256)
        res[name + "_x"], res[name + "_code"] = x, o.numpy()

    for case, (n, block, quant) in enumerate([(1000, 256, True), (300, 64, True), (1000, 256, False), (4096, 128, True)]):
        p = randn_bf16(rng, n, 0.02)
        g = randn_bf16(rng, n, 1e-3)
        gn = g.clone()
        if case == 0:
            gn[5] = float("inf"); gn[300] = float("nan"); gn[301] = float("-inf")
            gn[512:768] = 0.0     # a finite all-zero block
        if quant:
            s1 = torch.full((n,), 127, dtype=torch.uint8)
            s2 = torch.zeros(n, dtype=torch.uint8)
            a1 = torch.zeros(triton.cdiv(n, block)); a2 = torch.zeros_like(a1)
        else:
            s1 = torch.zeros(n, dtype=torch.bfloat16); s2 = torch.zeros(n, dtype=torch.bfloat16)
            a1 = a2 = p
        res[f"c{case}_p0"], res[f"c{case}_g"] = bits(p), bits(gn)
        q = p.clone()
        for step in (1, 2, 3):
            seed = (step * 2654435761 ^ (case + 3) * 1234567891) & 0xFFFFFFFF
            gg = gn if step == 1 else randn_bf16(rng, n, 1e-3)
            res[f"c{case}_g{step}"] = bits(gg)
            t8._adamw_8bit_kernel[(triton.cdiv(n, block),)](
                q, gg, s1, s2, a1, a2, Q1 if quant else q, Q2 if quant else q, n,
                1e-3, 0.9, 0.999, 1e-8, 0.01, 1 - 0.9 ** step, 1 - 0.999 ** step, seed,
                BLOCK=block, QUANTIZED=quant)
            res[f"c{case}_p{step}"] = bits(q)
            res[f"c{case}_s1_{step}"] = s1.numpy().copy() if quant else bits(s1)
            res[f"c{case}_s2_{step}"] = s2.numpy().copy() if quant else bits(s2)
            if quant:
                res[f"c{case}_a1_{step}"], res[f"c{case}_a2_{step}"] = a1.numpy().copy(), a2.numpy().copy()
            res[f"c{case}_seed{step}"] = np.uint64(seed)
        res[f"c{case}_meta"] = np.array([n, block, int(quant)])
    save("adamw8bit.npz", **res)

    # ---- Newton-Schulz (muon_sr.py:82-98) on CPU tensors ----
    res = {}
    shapes = [(2, 48, 80), (2, 80, 48), (1, 64, 64), (3, 24, 40), (1, 200, 96)]
    for k, shp in enumerate(shapes):
        x = randn_bf16(rng, int(np.prod(shp)), 1e-3).view(*shp)
        y = ms._newton_schulz(x, steps=5, out_dtype=None)
        res[f"x{k}"], res[f"y{k}"] = bits(x), bits(y)
        res[f"shape{k}"] = np.array(shp)
    save("newton_schulz.npz", count=np.array(len(shapes)), **res)

    # ---- whole optimizer trajectories through the reference's public classes ----
    def make_params(shapes, std, seed):
        r = np.random.default_rng(seed)
        return [torch.nn.Parameter(randn_bf16(r, int(np.prod(s)), std).view(*s)) for s in shapes]

    muon_shapes = [(24, 40), (24, 40), (40, 24), (24, 40), (40, 24), (16, 16)]
    adam_shapes = [(30, 16), (16,), (16,)]

    def run_hybrid(batch_ns, steps=4):
        mp = make_params(muon_shapes, 0.02, 1)
        ap = make_params(adam_shapes, 0.02, 2)
        opt = tm.TritonMuonSRWithAuxAdam([
            dict(params=mp, use_muon=True, lr=0.02, momentum=0.95, weight_decay=0.01),
            dict(params=ap, use_muon=False, lr=3e-4, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01),
        ], batch_ns=batch_ns)
        out = {"init_" + str(i): bits(p.detach()) for i, p in enumerate(mp + ap)}
        r = np.random.default_rng(3)
        for step in range(steps):
            for i, p in enumerate(mp + ap):
                drop = step == 2 and i in (1, 7)   # partial-grad step: one Muon, one AdamW param
                p.grad = None if drop else randn_bf16(r, p.numel(), 1e-3).view(p.shape)
                out[f"g{step}_{i}"] = np.zeros(0, np.uint16) if drop else bits(p.grad)
            opt.step()
            for i, p in enumerate(mp + ap):
                out[f"p{step}_{i}"] = bits(p.detach())
                st = opt.state[p]
                for key in ("momentum_buffer", "ema", "ema_squared"):
                    if key in st:
                        out[f"{key}{step}_{i}"] = bits(st[key])
                out[f"step{step}_{i}"] = np.array(st.get("step", -1))
        return out

    save("traj_hybrid_batch.npz", **run_hybrid(True))
    save("traj_hybrid_nobatch.npz", **run_hybrid(False))

    # TritonAdamW with gradient centralization (triton_adamw.py:117-203)
    ap = make_params([(12, 20), (20,)], 0.02, 4)
    opt = ta.TritonAdamW(ap, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, centralization=0.5)
    out = {"init_" + str(i): bits(p.detach()) for i, p in enumerate(ap)}
    r = np.random.default_rng(5)
    for step in range(3):
        for i, p in enumerate(ap):
            p.grad = randn_bf16(r, p.numel(), 1e-3).view(p.shape)
            out[f"g{step}_{i}"] = bits(p.grad)
        opt.step()
        for i, p in enumerate(ap):
            out[f"p{step}_{i}"] = bits(p.detach())
            out[f"ema{step}_{i}"] = bits(opt.state[p]["ema"])
            out[f"ema_squared{step}_{i}"] = bits(opt.state[p]["ema_squared"])
    save("traj_adamw_central.npz", **out)

    # TritonSRAccumulator: hooks draw seeds from Python's random module (triton_adamw.py:257)
    model = torch.nn.Sequential(torch.nn.Linear(16, 24), torch.nn.Linear(24, 8)).to(torch.bfloat16)
    with torch.no_grad():
        r = np.random.default_rng(6)
        for p in model.parameters():
            p.copy_(randn_bf16(r, p.numel(), 0.02).view(p.shape))
    out = {f"init_{i}": bits(p.detach()) for i, p in enumerate(model.parameters())}
    ta.TritonSRAccumulator.assign_hooks(model)
    random.seed(0)
    xb = randn_bf16(np.random.default_rng(7), 4 * 5 * 16, 1.0).view(4, 5, 16)
    out["x"] = bits(xb)
    for k in range(4):
        model(xb[k]).float().pow(2).mean().backward()
    for i, p in enumerate(model.parameters()):
        out[f"acc_{i}"] = bits(p.acc_grad)
    ta.TritonSRAccumulator.reassign_grad_buffer(model)
    for i, p in enumerate(model.parameters()):
        out[f"grad_{i}"] = bits(p.grad)
    save("traj_accum.npz", **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/muon_sr_checkout")
    main(sys.argv[1])
