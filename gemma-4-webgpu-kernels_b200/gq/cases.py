"""Named single-kernel workloads for profilers (one kernel family per case).

    python -m gq.cases <case> [--iters N]

Each case uploads synthetic weights at a BASELINE shape, runs a few warm-up calls
and then N calls of the one hot-path entry point, synchronised, so a profiler
can select launches of that kernel by name and skip the warm-up:

  config1   4-bit GEMV [6144, 1536], M = 1 (CUDA-core gemv_q_kernel); 64
            rotating weight copies so every call streams from HBM
  lm_head   I8 [262144, 1536] soft-capped GEMV, M = 1 (tensor-core gemv_tc_kernel)
  prefill   4-bit [6144, 1536] at M = 512 (cast_f16_kernel + prefill_tc_kernel)
  prefill_down  2-bit [1536, 6144] at M = 512, the config-3 down projection (K split
            over 4-CTA clusters)
  embed     config 4: 4096 ids into the 4-bit token table and the I8 PLE table
  embed_small  the same 4096 gathers from 32768-row tables (0.3 GB on the device,
            outputs 172 MB > L2): the case for multi-pass profiler captures
  decode    config 5: whole E2B decode steps (gq.e2b.Decoder, --batch sequences,
            2047-token cache); each "call" is one step (451 launches)
  attn      batch-64 attention over 2048 cached keys at head_dim 512 (ring kernel)
  tcx       8-row I8 GEMV [2048, 1536] (short-M tensor-core gemv_tcx_kernel)
  tcx_down  64-row 2-bit GEMV [1536, 6144], the batch-64 down projection (split-K
            over 4-CTA clusters)
  sample    gq_sample_rows on --batch rows of 262144 logits, temperature 1, top-k 64,
            top-p 0.95 (chunk top-k, chunk exp-sum, per-row candidate draw)

Run from the package directory (or with it on PYTHONPATH).
"""
from __future__ import annotations

import argparse
import sys
from ctypes import c_float, c_void_p


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["config1", "lm_head", "prefill", "prefill_down", "embed", "embed_small", "decode",
                                     "attn", "tcx", "tcx_down", "sample"])
    ap.add_argument("--iters", type=int, default=8)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)

    import numpy as np
    import torch

    from . import CudaBackend, synth

    g = CudaBackend(0)
    dev = g.torch_device
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    lib, ctx = g.lib, g.ctx

    def upload(n, k, bits, signed, seed):
        rb = k if signed else k * bits // 8
        payload = torch.randint(0, 256, (n * rb,), generator=gen, device=dev, dtype=torch.uint8)
        torch.cuda.synchronize()
        return g.quant_tensor_from_device(payload, synth.uniform(seed, n, 0.005, 0.02), (n, k), bits, signed, k)

    if args.case == "config1":
        ws = [upload(6144, 1536, 4, False, 100 + i) for i in range(64)]
        x = torch.randn(1, 1536, generator=gen, device=dev)
        y = torch.empty(1, 6144, device=dev)
        calls = [lambda w=w: lib.gq_linear(ctx, c_void_p(x.data_ptr()), 1, 1536, c_void_p(w.qw),
                                           c_void_p(y.data_ptr())) for w in ws]
    elif args.case == "lm_head":
        w = upload(synth.VOCAB, synth.HIDDEN, 8, True, 200)
        x = torch.randn(1, synth.HIDDEN, generator=gen, device=dev)
        y = torch.empty(1, synth.VOCAB, device=dev)
        calls = [lambda: lib.gq_linear_softcap(ctx, c_void_p(x.data_ptr()), 1, synth.HIDDEN, c_void_p(w.qw),
                                               c_float(30.0), c_void_p(y.data_ptr()), synth.VOCAB, 0)]
    elif args.case == "prefill":
        w = upload(6144, 1536, 4, False, 300)
        x = torch.randn(512, 1536, generator=gen, device=dev)
        y = torch.empty(512, 6144, device=dev)
        calls = [lambda: lib.gq_linear(ctx, c_void_p(x.data_ptr()), 512, 1536, c_void_p(w.qw),
                                       c_void_p(y.data_ptr()))]
    elif args.case == "prefill_down":
        w = upload(1536, 6144, 2, False, 310)
        x = torch.randn(512, 6144, generator=gen, device=dev)
        y = torch.empty(512, 1536, device=dev)
        calls = [lambda: lib.gq_linear(ctx, c_void_p(x.data_ptr()), 512, 6144, c_void_p(w.qw),
                                       c_void_p(y.data_ptr()))]
    elif args.case == "decode":
        from . import e2b

        dec = e2b.Decoder(g, e2b.e2b_config(), None, batch=args.batch, cache_len=2047, capacity=2048,
                          device_init_seed=5)
        dec.set_ids(np.arange(args.batch) * 4099 % synth.VOCAB)

        def step():
            dec.run()
            return 0
        calls = [step]
    elif args.case == "attn":
        from ._abi import GQ_ATTN_KPOS_IDENTITY

        b, s, dh = 64, 2048, 512
        q = torch.randn(b, 8, dh, generator=gen, device=dev)
        kc = torch.randn(b, s, dh, generator=gen, device=dev)
        vc = torch.randn(b, s, dh, generator=gen, device=dev)
        pos = torch.full((b,), s - 1, dtype=torch.int32, device=dev)
        out = torch.empty(b, 8 * dh, device=dev)
        calls = [lambda: lib.gq_attention(ctx, c_void_p(q.data_ptr()), b, 1, 8, dh, c_void_p(kc.data_ptr()),
                                          c_void_p(vc.data_ptr()), s, 1, s * dh, c_void_p(pos.data_ptr()), None, 0,
                                          c_float(1.0), 0, c_float(0.0), GQ_ATTN_KPOS_IDENTITY,
                                          c_void_p(out.data_ptr()))]
    elif args.case == "tcx":
        w = upload(2048, 1536, 8, True, 500)
        x = torch.randn(8, 1536, generator=gen, device=dev)
        y = torch.empty(8, 2048, device=dev)
        calls = [lambda: lib.gq_linear(ctx, c_void_p(x.data_ptr()), 8, 1536, c_void_p(w.qw),
                                       c_void_p(y.data_ptr()))]
    elif args.case == "tcx_down":
        w = upload(1536, 6144, 2, False, 600)
        x = torch.randn(64, 6144, generator=gen, device=dev)
        y = torch.empty(64, 1536, device=dev)
        calls = [lambda: lib.gq_linear(ctx, c_void_p(x.data_ptr()), 64, 6144, c_void_p(w.qw),
                                       c_void_p(y.data_ptr()))]
    elif args.case == "sample":
        import ctypes

        from . import _abi

        m = args.batch
        lg = torch.randn(m, synth.VOCAB, generator=gen, device=dev) * 3
        st = torch.arange(1, m + 1, dtype=torch.int64, device=dev)
        tok = torch.empty(m, dtype=torch.int32, device=dev)
        opts = _abi.SampleOpts(1.0, 64, 0.95, 1.0)
        calls = [lambda: lib.gq_sample_rows(ctx, c_void_p(lg.data_ptr()), m, synth.VOCAB, 0, ctypes.byref(opts),
                                            None, 0, 0, c_void_p(st.data_ptr()), c_void_p(tok.data_ptr()))]
    else:
        rows = synth.VOCAB if args.case == "embed" else 32768
        tok = upload(rows, synth.HIDDEN, 4, False, 400)
        rb = synth.LAYERS * synth.PLE_DIM
        payload = torch.randint(0, 256, (rows * rb,), generator=gen, device=dev, dtype=torch.uint8)
        torch.cuda.synchronize()
        ple = g.quant_tensor_from_device(payload, synth.uniform(401, rows * synth.LAYERS, 0.005, 0.02),
                                         (rows, rb), 8, True, synth.PLE_DIM)
        ids = torch.from_numpy(np.random.default_rng(4).integers(0, rows, 4096).astype(np.uint32)).to(dev)
        o1 = torch.empty(4096, synth.HIDDEN, device=dev)
        o2 = torch.empty(4096, rb, device=dev)
        calls = [lambda: (lib.gq_embed_rows(ctx, c_void_p(tok.qw), c_void_p(ids.data_ptr()), 4096,
                                            c_float(float(np.sqrt(synth.HIDDEN))), c_void_p(o1.data_ptr())),
                          lib.gq_embed_rows(ctx, c_void_p(ple.qw), c_void_p(ids.data_ptr()), 4096, c_float(16.0),
                                            c_void_p(o2.data_ptr())))]

    def run(n):
        for i in range(n):
            rc = calls[i % len(calls)]()
            for r in (rc if isinstance(rc, tuple) else (rc,)):
                if r != 0:
                    raise RuntimeError(f"{args.case}: status {r}")

    run(args.warmup)
    g.flush()
    run(args.iters)
    g.flush()
    g.close()
    print(f"{args.case}: {args.warmup} warm-up + {args.iters} calls ok")
    return 0


if __name__ == "__main__":
    sys.exit(main())
