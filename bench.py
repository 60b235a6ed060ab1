"""Benchmark of the activation-sparse ReLU^2 FFN hot path on B200.

Headline workload: one ReLU^2 FFN layer, forward + backward, d_model=4096,
d_ff=14336, 16384 tokens per GPU, bf16, up-projection bias shifted so that
90% of the activations are zero (the d=4096/14336 sparsity sweep).  Synthetic
seeded data: x ~ N(0,1), W_up ~ N(0, 1/4096), W_down ~ N(0, 1/14336),
upstream gradient ~ N(0,1).  Every tensor of a step is larger than L2 or is
rewritten each step, so no explicit L2 flush is used (inputs larger than L2).

Multi-GPU: one process per GPU (torchrun), tokens sharded (16384 per rank,
weak scaling); the only exchange is the NCCL all-reduce of dW1/dW2.

Also reported in the same JSON line: the dense cuBLAS bf16 FFN at the same
config, the sparsity sweep, standalone pack/unpack GB/s on [65536, 4096]
bf16 (p = 0.1), the 15-bit sign-strip codec (compress / uncompress GB/s at
3^16 bf16 values, and the reference harness's round-trip total over
n = 3^12..3^16), the roofline of the dominant kernel, and a CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

T_PER_GPU, D_MODEL, D_FF = 16384, 4096, 14336
SPARSITY = 0.9
SWEEP = (0.5, 0.8, 0.95, 0.99)
PACK_SHAPE, PACK_P = (65536, 4096), 0.1
PACK_SWEEP = (0.5, 0.2, 0.1, 0.05, 0.01)
CODEC_SIZES = tuple(3 ** i for i in range(12, 17))  # bitshifting/prepare.py:26
METRIC = "sparse FFN fwd+bwd tokens/s vs cuBLAS dense @80-95% sparsity; pack GB/s"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"],
                "bf16_tflops_sustained": p.get("bf16_tflops_sustained", p["bf16_tflops"]),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback"}


# ---------------------------------------------------------------- clocks ----
class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons while the timed region runs.
    Entering waits (up to 10 s) for nvidia-smi's first sample and then drops
    it, so that every kept sample falls inside the region (nvidia-smi takes a
    few hundred ms to start, longer than a short timed region)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            t0 = time.perf_counter()
            while not self.lines and self.proc.poll() is None and time.perf_counter() - t0 < 10.0:
                time.sleep(0.005)
            self.lines.clear()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=5)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# -------------------------------------------------------------- workload ----
def make_ffn_inputs(T, D, F, sparsity, device, seed=0):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(T, D, device=device, generator=g).to(torch.bfloat16)
    W1 = (torch.randn(F, D, device=device, generator=g) / D ** 0.5).to(torch.bfloat16)
    W2 = (torch.randn(D, F, device=device, generator=g) / F ** 0.5).to(torch.bfloat16)
    dout = torch.randn(T, D, device=device, generator=g).to(torch.bfloat16)
    b1 = torch.full((F,), bias_for_sparsity(x, W1, sparsity), device=device, dtype=torch.bfloat16)
    return x, W1, W2, b1, dout


def bias_for_sparsity(x, W1, s):
    """Scalar up-projection bias giving a fraction s of zeros after ReLU, from
    the quantile of the pre-activation on 1024 sampled tokens."""
    pre = (x[:1024] @ W1.T).float().flatten()
    return float(-torch.quantile(pre[:: max(1, pre.numel() // 8_000_000)], s))


# ------------------------------------------------ clustered sparsity ----
# The large ReLU^2 FFN sharded by tokens: d_model=8192, d_ff=28672, 8192
# tokens per GPU (65536 over 8), bf16.  Per 128-row token tile and 128-column
# cluster of d_ff the activation is entirely zero with p=0.5; elsewhere each
# entry is zero with p=0.8; non-zeros are |N(0,1)|.  The activation is
# injected (generated directly) and the step runs the layer's sparse part:
# the pack of z, the down-projection and the full backward.
CL_TOKENS, CL_D, CL_F = 8192, 8192, 28672


def clustered_activation(T, F, device, seed=0, p_cluster=0.5, p_zero=0.8):
    """bf16 [T, F]: 128x128 (token tile, column cluster) blocks zero with
    p_cluster, other entries zero with p_zero, non-zeros |N(0,1)| (an exact
    zero draw becomes the smallest normal, so the mask is the drawn one)."""
    g = torch.Generator(device=device).manual_seed(seed)
    dead = torch.rand(-(-T // 128), -(-F // 128), device=device, generator=g) < p_cluster
    dead = dead.repeat_interleave(128, 0)[:T].repeat_interleave(128, 1)[:, :F]
    keep = (torch.rand(T, F, device=device, generator=g) >= p_zero) & ~dead
    del dead
    v = torch.randn(T, F, device=device, generator=g).abs_().clamp_min_(torch.finfo(torch.bfloat16).tiny)
    return torch.where(keep, v, 0.0).to(torch.bfloat16)


def make_clustered_inputs(T, D, F, device, seed=0):
    """x ~ N(0,1) [T, D], W1 ~ N(0,1/D) [F, D], W2 ~ N(0,1/F) [D, F], the
    clustered activation z [T, F] and dout ~ N(0,1) [T, D], all bf16."""
    g = torch.Generator(device=device).manual_seed(seed + 1000)
    x = torch.randn(T, D, device=device, generator=g).to(torch.bfloat16)
    W1 = (torch.randn(F, D, device=device, generator=g) / D ** 0.5).to(torch.bfloat16)
    W2 = (torch.randn(D, F, device=device, generator=g) / F ** 0.5).to(torch.bfloat16)
    dout = torch.randn(T, D, device=device, generator=g).to(torch.bfloat16)
    return x, W1, W2, clustered_activation(T, F, device, seed), dout


class ClusteredStep:
    """The sparse part of one ReLU^2 FFN layer on an injected activation:
    dense_to_tilesparse(z) into the arena, the down-projection from the packed
    z and the backward (dX, dW1, dW2; weight gradients all-reduced under data
    parallelism), through the public API."""

    def __init__(self, x, W1, W2, z, dout, group=None):
        import autoresearch2_b200 as sf
        self.sf = sf
        self.x, self.W1, self.W2, self.z, self.dout = x, W1, W2, z, dout
        self.comm = sf.parallel.GradAllReduce(group) if group is not None else None
        T, F = z.shape
        self.buf = sf.TensorBuffer(T * F // 2, z.device, z.dtype).init_buffer()

    def packed(self):
        self.buf.reset_buffer()
        vals, off = self.buf.as_sparse_data()
        return self.sf.dense_to_tilesparse(self.z, vals, off, 128, 128)

    def __call__(self):
        zs = self.packed()
        out = self.sf.ffn.down_proj(zs, self.W2)
        if self.comm is None:
            grads = self.sf.ffn.packed_backward(self.dout, self.x, self.W1, self.W2, zs)
        else:
            with self.comm.attached():
                grads = self.sf.ffn.packed_backward(self.dout, self.x, self.W1, self.W2, zs)
            self.comm.wait()
        return out, grads


class ClusteredDenseStep:
    """The same products dense on cuBLAS bf16: out = bf16(z^2) @ W2^T and the
    backward of FFNrelu2 from dZ (old/lib_sparse/prepare_layer.py:12-29)."""

    def __init__(self, x, W1, W2, z, dout):
        self.x, self.W1, self.W2, self.z, self.dout = x, W1, W2, z, dout

    def __call__(self):
        a = self.z * self.z
        out = a @ self.W2.T
        dW2 = self.dout.T @ a
        dpre = (self.dout @ self.W2) * 2 * self.z
        dW1 = dpre.T @ self.x
        dx = dpre @ self.W1
        return out, (dx, dW1, dW2)


def bench_clustered(device, group, world, steps, warmup, pk, rank):
    """The clustered-sparsity leg: tokens/s of ClusteredStep (8192 tokens per
    GPU, weak scaling) on the auto-chosen path, the two paths forced, the live
    fraction of (tile, column) pairs, and on one GPU the dense cuBLAS step."""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import gemm as G
    T, D, F = CL_TOKENS, CL_D, CL_F
    x, W1, W2, z, dout = make_clustered_inputs(T, D, F, device, seed=rank)
    step = ClusteredStep(x, W1, W2, z, dout, group)
    res = {"workload": f"relu2_ffn_clustered_d{D}_f{F}_t{T}", "tokens_per_gpu": T, "global_tokens": T * world,
           "d_model": D, "d_ff": F}
    zs = step.packed()
    kc = G.ck_lists(G.tile_colmask(zs), T, F, counts_only=True)[1]
    kp = ((kc.long() + 63) // 64 * 64).sum().item()
    live = kc.sum().item() / (T // 128 * F)
    res["zeros"] = round(1 - int(zs.prefix[-1].item()) / (T * F), 4)
    res["live_column_fraction"] = round(live, 4)
    res["executed_k_fraction"] = round(kp / (T // 128 * F), 4)
    mode = sf.compact_k()
    for name, m in (("auto", mode), ("dense_k", "off"), ("compacted_k", "on")):
        sf.set_compact_k(m)
        ms = time_steps(step, steps, max(warmup, 3), device)
        res[name] = {"tokens_per_s": round(T * world / (ms / 1e3), 1), "ms_per_step": round(ms, 3),
                     "path": sf.ffn.last_path()}
    sf.set_compact_k(mode)
    base = 2.0 * T * D * F
    ms = res["auto"]["ms_per_step"]
    res["flops"] = {"dense_equivalent_per_step": 5 * base, "executed_compacted_per_step":
                    base * (3 + 2 * kp / (T // 128 * F)),
                    "algorithmic_per_step": 5 * base * (1 - res["zeros"]),
                    "dense_equivalent_tflops": round(5 * base / (ms * 1e-3) / 1e12, 1)}
    if world == 1:
        dense = ClusteredDenseStep(x, W1, W2, z, dout)
        dms = time_steps(dense, steps, max(warmup, 3), device)
        res["dense_cublas"] = {"tokens_per_s": round(T / (dms / 1e3), 1), "ms_per_step": round(dms, 3)}
        res["speedup_vs_dense"] = round(dms / ms, 3)
        del dense
    del step, x, W1, W2, z, dout, zs
    torch.cuda.empty_cache()
    sf.check_status(device)
    return res


class Step:
    """One forward + backward of the sparse ReLU^2 FFN through the public API."""

    def __init__(self, x, W1, W2, b1, dout, group=None):
        import autoresearch2_b200 as sf
        self.sf = sf
        self.comm = sf.parallel.GradAllReduce(group) if group is not None else None
        self.x, self.dout = x, dout
        self.W1 = W1.clone().requires_grad_()
        self.W2 = W2.clone().requires_grad_()
        self.b1 = b1.clone().requires_grad_()
        T, F = x.shape[0], W1.shape[0]
        self.buf = sf.TensorBuffer(T * F, x.device, x.dtype).init_buffer()
        self.group = group

    def __call__(self, x=None, dout=None):
        x = self.x if x is None else x
        dout = self.dout if dout is None else dout
        self.buf.reset_buffer()
        for p in (self.W1, self.W2, self.b1):
            p.grad = None
        out = self.sf.FFNSpRelu2.apply(x, self.W1, self.W2, self.buf.as_sparse_data(), self.b1)
        if self.comm is None:
            out.backward(dout)
        else:
            # dW sums over the token shards overlap the rest of the backward
            with self.comm.attached():
                out.backward(dout)
            self.comm.wait()
        return out


class DenseStep:
    """Dense cuBLAS bf16 ReLU^2 FFN, autograd of the reference's FFNrelu2
    (old/lib_sparse/prepare_layer.py:12-29) plus the bias."""

    def __init__(self, x, W1, W2, b1, dout):
        self.x, self.dout = x, dout
        self.W1 = W1.clone().requires_grad_()
        self.W2 = W2.clone().requires_grad_()
        self.b1 = b1.clone().requires_grad_()

    def __call__(self):
        for p in (self.W1, self.W2, self.b1):
            p.grad = None
        z = torch.relu(self.x @ self.W1.T + self.b1) ** 2
        out = z @ self.W2.T
        out.backward(self.dout)
        return out


def time_steps(fn, steps, warmup, device):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize(device)
    if dist.is_initialized():
        dist.barrier()
    ms = a.elapsed_time(b)
    if dist.is_initialized():
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms / steps


# ------------------------------------------------------------------ pack ----
def bench_pack(device, p=PACK_P, reps=20):
    """Flat pack and unpack of a [65536, 4096] bf16 tensor whose entries are
    nonzero with probability p (|N(0,1)| + 1e-3), timed through the C ABI with
    preallocated buffers: median over `reps` calls of CUDA-event time on the
    launching stream.  Each call reads or writes 537 MB of dense data, more
    than L2, so no flush is needed.  Round trip checked bit-exact."""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import _lib
    rows, cols = PACK_SHAPE
    g = torch.Generator(device=device).manual_seed(0)
    keep = torch.rand(rows, cols, device=device, generator=g) < p
    d = torch.where(keep, torch.randn(rows, cols, device=device, generator=g).abs() + 1e-3,
                    torch.zeros((), device=device)).to(torch.bfloat16)
    del keep
    n = d.numel()
    vals, mask = sf.bitsparse_pack(d)
    nnz = vals.numel()
    algo = 2 * n + n / 8 + 2 * nnz  # bytes moved per pack (and per unpack)
    L = _lib.load()
    vbuf = torch.empty(n, dtype=d.dtype, device=device)
    nnz_d = torch.zeros(2, dtype=torch.int64, device=device)
    ws = _lib.workspace(L.sffn_flat_pack_workspace_bytes(n, _lib.BF16), device)
    out = torch.empty_like(d)
    st = _lib.stream_ptr(device)
    status = _lib.status_word(device)

    def pack():
        _lib.call("sffn_flat_pack", _lib.ptr(d), 1, n, _lib.ptr(mask), _lib.ptr(vbuf), n,
                  _lib.ptr(nnz_d), _lib.ptr(ws), ws.numel(), _lib.ptr(status), st)

    def unpack():
        _lib.call("sffn_flat_unpack", _lib.ptr(vals), nnz, _lib.ptr(mask), 1, n, _lib.ptr(out),
                  _lib.ptr(ws), ws.numel(), _lib.ptr(status), st)

    res = {}
    for name, fn in (("pack", pack), ("unpack", unpack)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(device)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * reps)]
        for i in range(reps):
            ev[2 * i].record()
            fn()
            ev[2 * i + 1].record()
        torch.cuda.synchronize(device)
        ms = statistics.median(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(reps))
        res[name] = {"gbs": algo / ms / 1e6, "ms": ms}
    _lib.check_status(device)
    assert torch.equal(out, d)
    assert int(nnz_d[0]) == nnz and torch.equal(vbuf[:nnz], vals)
    return {"shape": list(PACK_SHAPE), "p": p, "dtype": "bf16", "algo_bytes": algo,
            "pack_gbs": round(res["pack"]["gbs"], 1), "unpack_gbs": round(res["unpack"]["gbs"], 1),
            "pack_ms": round(res["pack"]["ms"], 4), "unpack_ms": round(res["unpack"]["ms"], 4)}


# ----------------------------------------------------------- codec15 ----
def bench_codec15(device, reps=20, iters=100):
    """The 15-bit sign-strip codec on |N(0,1)| bf16 data (bitshifting/prepare.py:8-10).

    Kernels: compress and uncompress of 3^16 values through the C ABI with
    preallocated buffers; median over `reps` calls of CUDA-event time on the
    launching stream, L2 flushed (a 256 MB buffer zeroed) before each call,
    since the 86 MB of data fit in L2.  GB/s = (2 n + ceil(15 n / 8)) / time.
    Harness: the reference's figure -- for each n in 3^12..3^16, the mean of
    `iters` compress_fn + uncompress_fn round trips through the public API
    after 5 warm-up ones (prepare.py:29-49), summed over the sizes; checked
    exact like prepare.py:45."""
    from autoresearch2_b200 import _lib, bitshift
    g = torch.Generator(device=device).manual_seed(0)
    n = CODEC_SIZES[-1]
    x = torch.randn(n, generator=g, device=device).to(torch.bfloat16).abs()
    nb = bitshift.compressed_bytes(n)
    stream = torch.empty(bitshift.padded_bytes(n), dtype=torch.uint8, device=device)
    back = torch.empty_like(x)
    flush = torch.empty(256 * 2 ** 20, dtype=torch.uint8, device=device)
    st = _lib.stream_ptr(device)

    def compress():
        _lib.call("sffn_codec15_compress", _lib.ptr(x), n, _lib.ptr(stream), stream.numel(), st)

    def uncompress():
        _lib.call("sffn_codec15_uncompress", _lib.ptr(stream), stream.numel(), n, _lib.ptr(back), st)

    algo = 2 * n + nb
    res = {"n": n, "algo_bytes": algo}
    for name, fn in (("compress", compress), ("uncompress", uncompress)):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(reps):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b))
        ms = statistics.median(ts)
        res[f"{name}_gbs"] = round(algo / ms / 1e6, 1)
        res[f"{name}_ms"] = round(ms, 4)
    assert torch.equal(back, x)
    del flush
    total = 0.0
    for m in CODEC_SIZES:
        d = torch.randn(m, generator=g, device=device).to(torch.bfloat16).abs()
        for _ in range(5):
            bitshift.uncompress_fn(bitshift.compress_fn(d), d.shape, torch.bfloat16)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            out = bitshift.uncompress_fn(bitshift.compress_fn(d), d.shape, torch.bfloat16)
        b.record()
        b.synchronize()
        assert torch.equal(out, d)
        total += a.elapsed_time(b) / iters
    res["harness_total_ms"] = round(total, 4)
    res["harness_sizes"] = list(CODEC_SIZES)
    return res


# -------------------------------------------------------------- deep ----
def bench_deep(device):
    """The reference's multi-layer harness (old/lib_sparse/prepare.py:115-148):
    4 residual ReLU FFN layers, width 4096, hidden 21504, 10000 tokens, bf16,
    Xavier weights; dense baseline (dense ReLU output kept per layer) against
    the sparse stack over one arena of 0.55 x the dense activation size.
    Peak MB from torch's allocator, ms per step by host clock around
    synchronised steps (as the harness); eager, no torch.compile.  Also the
    same report at the model's default depth of 12 layers (prepare.py:51),
    where the arena's saving outgrows the fused path's per-layer transients."""
    from autoresearch2_b200 import deep
    g = torch.Generator(device=device).manual_seed(0)
    x = torch.randn(10000, 4096, generator=g, device=device, dtype=torch.bfloat16)
    model = deep.DeepFFN(torch.bfloat16, layers=4, hidm=4096, device=device)
    r = deep.memory_report(x, model)
    del model
    torch.cuda.empty_cache()
    model = deep.DeepFFN(torch.bfloat16, layers=12, hidm=4096, device=device)
    r12 = deep.memory_report(x, model)
    r["layers_12"] = {k: r12[k] for k in ("resident_mb", "dense", "sparse", "sparse_exact", "arena",
                                          "loss_rel_diff")}
    del model, x
    torch.cuda.empty_cache()
    return r


# --------------------------------------------------------------- gpt ----
def bench_gpt(device, pk, steps=5, warmup=3, world=1, rank=0):
    """GPT-style training step with the sparse ReLU^2 MLPs against the same
    model with dense torch MLPs: 12 layers, width 768, 12 heads, hidden 3072,
    vocab 50304, 1024-token sequences, batch 32 per GPU (32768 tokens per
    GPU per step), bf16, N(0, 0.02) weights, uniform random token ids (seed
    0 + rank), fused AdamW; with N GPUs data-parallel (torch's
    DistributedDataParallel over NCCL, weak scaling).  Whole-job tokens/s from
    CUDA events over `steps` steps after `warmup`, max over ranks; MFU per GPU
    against the measured sustained bf16 figure; peak MB from torch's allocator."""
    from autoresearch2_b200 import gpt
    cfg = gpt.GPTConfig()
    batch = 32
    idx, tgt = gpt.synthetic_batch(cfg, batch, device, seed=rank)
    res = {"config": {"n_layer": cfg.n_layer, "n_embd": cfg.n_embd, "n_head": cfg.n_head,
                      "ffn_hidden": cfg.ffn_hidden, "vocab": cfg.vocab, "seq_len": cfg.seq_len,
                      "batch": batch, "mlp": "relu2"},
           "flops_per_token": gpt.flops_per_token(cfg)}
    res["n_gpus"] = world
    for name, sparse in (("sparse", True), ("dense", False)):
        model = gpt.GPT(cfg, sparse=sparse, device=device)
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[device.index]) if world > 1 else model
        step = gpt.TrainStep(net, idx, tgt)
        torch.cuda.reset_peak_memory_stats(device)
        ms = time_steps(step, steps, warmup, device)
        loss = float(step())
        tps = world * batch * cfg.seq_len / (ms / 1e3)
        res[name] = {"tokens_per_s": round(tps, 1), "ms_per_step": round(ms, 3),
                     "mfu_of_measured_sustained": round(gpt.mfu(tps / world, cfg, pk["bf16_tflops_sustained"]), 3),
                     "peak_mb": round(torch.cuda.max_memory_allocated(device) / 2 ** 20, 1),
                     "loss_after": round(loss, 4)}
        if sparse:
            res[name]["activation_zeros"] = round(
                1 - model.arena.used() / (batch * cfg.seq_len * cfg.ffn_hidden * cfg.n_layer), 4)
        del step, net, model
        torch.cuda.empty_cache()
    import autoresearch2_b200 as sf
    sf.check_status(device)
    return res


# ---------------------------------------------------------- CPU baseline ----
class _HostThreads:
    """Every host core for torch's and BLAS's thread pools while a CPU leg
    runs, whatever OMP_NUM_THREADS a launcher set (torchrun sets 1)."""

    def __enter__(self):
        self.cores = os.cpu_count() or 1
        self.prev = torch.get_num_threads()
        torch.set_num_threads(self.cores)
        self.limiter = None
        try:
            from threadpoolctl import threadpool_limits
            self.limiter = threadpool_limits(limits=self.cores)
        except Exception:  # noqa: BLE001
            pass
        return self

    def __exit__(self, *exc):
        torch.set_num_threads(self.prev)
        if self.limiter is not None:
            self.limiter.restore_original_limits()


def _cpu_flat_round_trip(z):
    """The flat pack and unpack of z on the host (the C restatement of the
    reference's bit order, old/bitpack/prepare.py:6-23), checked exact."""
    import numpy as np
    import oracle
    zn = z.detach().contiguous().numpy()
    vals, mask = oracle.flat_pack(zn, nthreads=os.cpu_count() or 1)
    back = oracle.flat_unpack(vals, mask, zn.shape, nthreads=os.cpu_count() or 1)
    assert np.array_equal(back.view(np.uint32), zn.view(np.uint32))
    return vals.size


def cpu_reference_ffn(T, D, F, steps, warmup, sparsity=None, bias=None, seed=0):
    """The reference's dense torch ReLU^2 FFN on the host cores: FFNrelu2
    (old/lib_sparse/prepare_layer.py:12-29: relu(x @ W1.T)^2 @ W2.T, here with
    the up-projection bias) forward and torch autograd backward in float32,
    then the flat pack/unpack round trip of z, `warmup` untimed and `steps`
    timed steps.  x ~ N(0,1), W1 ~ N(0,1/D), W2 ~ N(0,1/F), dout ~ N(0,1),
    seeded; the bias is `bias`, or the quantile giving `sparsity` zeros."""
    with _HostThreads() as ht:
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(T, D, generator=g)
        W1 = (torch.randn(F, D, generator=g) / D ** 0.5).requires_grad_()
        W2 = (torch.randn(D, F, generator=g) / F ** 0.5).requires_grad_()
        dout = torch.randn(T, D, generator=g)
        if bias is None:
            with torch.no_grad():
                pre = (x[:256] @ W1.T).flatten()
                bias = float(-torch.quantile(pre[:: max(1, pre.numel() // 8_000_000)], sparsity))
        b1 = torch.full((F,), float(bias)).requires_grad_()
        nnz = [0]

        def step():
            for p in (W1, W2, b1):
                p.grad = None
            z = torch.relu(x @ W1.T + b1)
            out = (z ** 2) @ W2.T
            out.backward(dout)
            nnz[0] = _cpu_flat_round_trip(z)

        for _ in range(warmup):
            step()
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        dt = time.perf_counter() - t0
        return {"value": round(steps * T / dt, 1), "unit": "tokens/s", "cores": ht.cores,
                "torch_threads": torch.get_num_threads(), "nproc": os.cpu_count(),
                "ms_per_step": round(dt / steps * 1e3, 2), "bias": round(float(bias), 5),
                "measured_sparsity": round(1 - nnz[0] / (T * F), 4), "kind": "port",
                "sample": f"{steps} x {T} tokens of the D={D}, F={F} ReLU^2 FFN fwd+bwd (torch float32, "
                          f"FFNrelu2 + autograd) + flat pack/unpack round trip of z, after {warmup} "
                          f"untimed; {dt:.1f} s"}


def cpu_oracle_port(sample_tokens, steps=1, warmup=0):
    """The oracle (numpy restatement of the reference's dense ReLU^2 FFN and
    the C restatement of its tiled pack) on the host cores: `warmup` untimed
    and `steps` timed samples of `sample_tokens` tokens of the headline
    workload.  Returns tokens/s over the timed samples."""
    import numpy as np
    import oracle
    with _HostThreads() as ht:
        rng = np.random.default_rng(0)
        T, D, F = sample_tokens, D_MODEL, D_FF
        x = rng.standard_normal((T, D), dtype=np.float32)
        W1 = (rng.standard_normal((F, D), dtype=np.float32) / np.sqrt(D)).astype(np.float32)
        W2 = (rng.standard_normal((D, F), dtype=np.float32) / np.sqrt(F)).astype(np.float32)
        dout = rng.standard_normal((T, D), dtype=np.float32)
        pre = x @ W1.T
        b1 = np.full(F, -np.quantile(pre[:256], SPARSITY), dtype=np.float32)
        arena = np.empty(T * F, dtype=np.float32)

        def sample():
            r = oracle.ffn_fwd_bwd(x, W1, W2, dout, act="relu2", b1=b1, code=oracle.F32,
                                   compute=np.float32)
            oracle.tile_pack(r["z"].astype(np.float32), 128, 128, arena, 0)

        for _ in range(warmup):
            sample()
        t0 = time.perf_counter()
        for _ in range(steps):
            sample()
        dt = time.perf_counter() - t0
        return {"value": round(steps * T / dt, 1), "unit": "tokens/s", "cores": ht.cores, "kind": "port",
                "sample": f"{steps} x {T} tokens of the d=4096/14336 ReLU^2 FFN fwd+bwd (float32 numpy) "
                          f"+ tiled pack of z, after {warmup} untimed; {dt:.1f} s"}


# configs[0]-style single layer on the CPU: T=8192 (8 x 1024), D=768, F=3072,
# float32, up-projection bias -1.3 (about 90% zeros)
CFG1 = {"T": 8192, "D": 768, "F": 3072, "bias": -1.3}


def cpu_baselines(sample_tokens, steps, warmup):
    """The CPU figures of the bench line: the reference's dense torch path at
    the headline shape on a token sample (the baseline proper), at the exact
    single-layer CPU configuration, and the numpy/C oracle port."""
    base = cpu_reference_ffn(sample_tokens, D_MODEL, D_FF, steps, warmup, sparsity=SPARSITY)
    base["cfg1"] = cpu_reference_ffn(CFG1["T"], CFG1["D"], CFG1["F"], 3, 1, bias=CFG1["bias"])
    base["cfg1"]["config"] = dict(CFG1, dtype="f32")
    base["oracle_port"] = cpu_oracle_port(sample_tokens, steps=4, warmup=1)
    return base


def workload_config(tpg, world, tokens, s_meas=None):
    """The `config` of both arms' lines."""
    c = {"workload": f"relu2_ffn_fwd_bwd_d4096_f14336_t{tpg}_s0.9", "tokens_per_gpu": tpg,
         "global_tokens": tokens, "d_model": D_MODEL, "d_ff": D_FF, "target_sparsity": SPARSITY,
         "parallelism": f"dp{world}", "l2": "inputs larger than L2"}
    if s_meas is not None:
        c["measured_sparsity"] = round(s_meas, 4)
    return c


# -------------------------------------------------------------- roofline ----
# DRAM traffic per launch of the roofline kernels at T=16384: dram__bytes_read.sum
# + dram__bytes_write.sum of one ncu capture of each kernel at that size
# (bench.py --micro up / dgrad: up 1105 + 534 MB, activation gradient 1366 + 908 MB).
TRAFFIC_BYTES = {"sffn_ffn_up": 1105e6 + 534e6, "sffn_ffn_dgrad": 1366e6 + 908e6}


def kernel_breakdown(timer, steps_recorded, step_ms):
    """Per C-ABI entry point: launches per step, mean device ms per launch (CUDA
    events on the launching stream over warm-up + timed steps) and its share
    of the step time."""
    out = {}
    for name, v in sorted(timer.summary().items(), key=lambda kv: -kv[1]["total_ms"]):
        per_step = v["calls"] / steps_recorded
        out[name] = {"launches_per_step": round(per_step, 2), "mean_ms": round(v["mean_ms"], 4),
                     "share_of_step": round(v["mean_ms"] * per_step / step_ms, 3)}
    return out


def roofline(kernels, tokens, pk, s=SPARSITY):
    """Tensor-core roofline of the largest single launch of the step.

    The fused up-projection (x @ W1^T with the ReLU^2/bitmask epilogue) and the
    fused activation-gradient GEMM (dout @ W2 with the ReLU^2 derivative) each
    execute 2*T*D*F flops.  Their algorithmic work differs: the up-projection
    is dense (the sparsity is only known after it), while the activation
    gradient is only needed at the live entries of z, 2*T*D*F*(1 - s).
    `achieved` and `frac` count the algorithmic flops; `executed_*` count the
    flops the kernel runs.  The denominator is the sustained cuBLAS bf16
    figure, as both kernels run inside a long step at the power cap."""
    cands = [k for k in ("sffn_ffn_dgrad", "sffn_ffn_up") if k in kernels]
    if not cands:
        return None
    name = max(cands, key=lambda k: kernels[k]["mean_ms"])
    executed = 2.0 * tokens * D_MODEL * D_FF
    algo = executed if name == "sffn_ffn_up" else executed * (1.0 - s)
    ms = kernels[name]["mean_ms"]
    tf = algo / (ms * 1e-3) / 1e12
    etf = executed / (ms * 1e-3) / 1e12
    peak = pk["bf16_tflops_sustained"]
    return {"bound": "tensor", "kernel": name, "achieved": round(tf, 1), "peak": peak,
            "unit": "TFLOP/s", "frac": round(tf / peak, 4), "traffic": TRAFFIC_BYTES.get(name),
            "algorithmic_flops_per_launch": algo, "executed_flops_per_launch": executed,
            "executed_achieved": round(etf, 1), "executed_frac": round(etf / peak, 3),
            "sparsity": round(s, 4), "ms_per_launch": ms,
            "peak_source": f"{pk['source']} (sustained bf16)"}


def step_flops(step, ms, s, pk):
    """The step's FLOPs three ways, per GPU: dense-equivalent 12 T D F; the
    algorithmic sparse count 2 T D F (1 + 5 (1 - s)) (the up-projection dense,
    the down-projection, dgrad's live entries, dW2, dX and dW1 scaling with
    the nonzeros); and what the kernels execute, 2 T D F (4 + 2 l) with l the
    fraction of 64-wide K blocks that are live in a 256-row tile (the
    down-projection and dX skip the others; the up-projection, the
    activation-gradient GEMM, dW1 and dW2 run dense).  l is read from one
    more forward's K-block lists; rates use the step time `ms`."""
    import autoresearch2_b200 as sf
    T, D = step.x.shape
    F = step.W1.shape[0]
    step.buf.reset_buffer()
    out = sf.FFNSpRelu2.apply(step.x, step.W1, step.W2, step.buf.as_sparse_data(), step.b1)
    kb_count = out.grad_fn.aux[2]
    nkb = -(-F // 64)
    live = float(kb_count.sum()) / (kb_count.numel() * nkb) if kb_count.numel() else None
    path = sf.ffn.last_path()
    del out
    base = 2.0 * T * D * F
    dense_eq, alg = 6 * base, base * (1 + 5 * (1 - s))
    exe = base * (4 + 2 * live) if live is not None else None
    rate = lambda f: round(f / (ms * 1e-3) / 1e12, 1)  # noqa: E731
    r = {"dense_equivalent_per_step": dense_eq, "algorithmic_per_step": alg,
         "live_kblock_fraction": None if live is None else round(live, 4), "products_path": path,
         "dense_equivalent_tflops": rate(dense_eq), "algorithmic_tflops": rate(alg),
         "algorithmic_frac_of_measured_sustained": round(alg / (ms * 1e-3) / 1e12 / pk["bf16_tflops_sustained"], 4),
         "peak_tflops": pk["bf16_tflops_sustained"]}
    if exe is not None:
        r["executed_per_step"] = exe
        r["executed_tflops"] = rate(exe)
        r["executed_frac_of_measured_sustained"] = round(exe / (ms * 1e-3) / 1e12 / pk["bf16_tflops_sustained"], 3)
    return r


# ------------------------------------------------------------ micro ----
def micro(case, device, reps=3):
    """A few launches of one group of kernels at a stated size, for kernel
    timing and profiler captures; prints one JSON line of CUDA-event times
    (mean ms per call after one warm-up call).
      flat   flat pack and unpack, [65536, 4096] bf16, p = 0.1
      tile   tiled pack (128 x 128) and unpack of the clustered activation
             [8192, 28672] bf16, plus the per-row offsets of its tiles
      up     the fused up-projection GEMM (+ tile scan and slot gather) of the
             headline layer, `tokens` tokens, 90% zeros
      dgrad  the fused activation-gradient GEMM of the same layer
      ck     the compacted-K GEMM of the clustered workload's down-projection
      relu_ax  relu(x @ W1.T) at old/matmul_bitsparse's largest harness shape
             (x [10000, 4096], W1 [16384, 4096], shifted inputs): the float32
             kind::tf32 GEMM alone (ReLU in the epilogue), then the whole of
             tiled.sparse_relu_Ax in float32 and in bf16 (the fused
             up-projection)"""
    import autoresearch2_b200 as sf
    from autoresearch2_b200 import _lib, gemm as G, sp24
    res = {"case": case}

    def run(name, fn):
        fn()
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize(device)
        res[name + "_ms"] = round(a.elapsed_time(b) / reps, 4)

    if case == "flat":
        g = torch.Generator(device=device).manual_seed(0)
        d = torch.where(torch.rand(*PACK_SHAPE, device=device, generator=g) < PACK_P,
                        torch.randn(*PACK_SHAPE, device=device, generator=g).abs() + 1e-3, 0.0).to(torch.bfloat16)
        vals, mask = sf.bitsparse_pack(d)
        run("pack", lambda: sf.bitsparse_pack_async(d, torch.empty_like(d).view(-1)))
        run("unpack", lambda: sf.bitsparse_unpack(vals, mask, d.shape))
    elif case == "tile":
        z = clustered_activation(CL_TOKENS, CL_F, device)
        arena = torch.empty(z.numel() // 2, dtype=z.dtype, device=device)
        off = torch.zeros(1, dtype=torch.int32, device=device)

        def pk():
            off.zero_()
            return sf.dense_to_tilesparse(z, arena, off, 128, 128)
        zs = pk()
        run("tile_pack", pk)
        run("tile_unpack", lambda: sf.tile_unpack(zs))
        run("tile_row_offsets", lambda: G.tile_row_offsets(zs))
    elif case in ("up", "dgrad"):
        x, W1, W2, b1, dout = make_ffn_inputs(micro.tokens, D_MODEL, D_FF, SPARSITY, device)
        arena = torch.empty(micro.tokens * D_FF, dtype=torch.bfloat16, device=device)
        off = torch.zeros(1, dtype=torch.int32, device=device)

        def up():
            off.zero_()
            return G.ffn_up(x, W1, b1, G.ACT_RELU2, arena, off)
        _, bm, pf, vo, ro = up()
        zs = sf.BitsparseTensor(arena, bm, pf, vo, -(-micro.tokens // 128), D_FF // 128, 128, 128,
                                (micro.tokens, D_FF))
        if case == "up":
            run("ffn_up", up)
        else:
            run("ffn_dgrad", lambda: G.ffn_dgrad(dout, W2, G.ACT_RELU2, zs, ro))
    elif case == "ck":
        x, W1, W2, z, dout = make_clustered_inputs(CL_TOKENS, CL_D, CL_F, device)
        arena = torch.empty(z.numel() // 2, dtype=z.dtype, device=device)
        off = torch.zeros(1, dtype=torch.int32, device=device)
        zs = sf.dense_to_tilesparse(z, arena, off, 128, 128)
        cm = G.tile_colmask(zs)
        idx, kc, cp = G.ck_lists(cm, CL_TOKENS, CL_F)
        ac = G.ck_gather_packed(zs, G.tile_row_offsets(zs), cm, cp, kc, G.ACT_RELU2)
        W2t = sp24.transpose(W2)
        run("gemm_ck", lambda: G.ck_mm(ac, W2t, idx, kc))
    elif case == "relu_ax":
        g = torch.Generator(device=device).manual_seed(1)
        rows, tokens = 4096, 10000
        W1 = torch.empty(4 * rows, rows, device=device)
        torch.nn.init.xavier_uniform_(W1, generator=g)
        x = torch.randn(tokens, rows, device=device, generator=g)
        W1, x = W1 + 0.1 * W1.std(), x - 0.1 * x.std()
        run("gemm_tf32", lambda: G.matmul_tf32(x, W1, relu=True))
        res["gemm_tf32_tflops"] = round(2.0 * tokens * rows * 4 * rows / res["gemm_tf32_ms"] / 1e9, 1)
        run("sparse_relu_Ax_f32", lambda: sf.tiled.sparse_relu_Ax(W1, x))
        W1b, xb = W1.bfloat16(), x.bfloat16()
        run("sparse_relu_Ax_bf16", lambda: sf.tiled.sparse_relu_Ax(W1b, xb))
    else:
        raise SystemExit(f"unknown micro case {case}")
    sf.check_status(device)
    print(json.dumps(res), flush=True)


micro.tokens = T_PER_GPU


# ------------------------------------------------------------------ main ----
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=1024)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-clustered", action="store_true",
                    help="skip the clustered-sparsity large-FFN leg (d=8192/28672)")
    ap.add_argument("--tokens", type=int, default=T_PER_GPU,
                    help="tokens per GPU (smaller cases are for profiling)")
    ap.add_argument("--quick", action="store_true",
                    help="time the sparse step only: no dense, sweep, e2e, pack or CPU legs")
    ap.add_argument("--pack-only", action="store_true",
                    help="only the flat pack/unpack sweep over p (one JSON line per p)")
    ap.add_argument("--sparse-mma", default="auto", choices=["auto", "on", "off"],
                    help="path of the products with a sparse operand: 2:4 sparse tensor cores "
                         "chosen by the observed sparsity (auto), always, or never")
    ap.add_argument("--micro", choices=["flat", "tile", "up", "dgrad", "ck", "relu_ax"],
                    help="time one group of kernels at a stated size (and nothing else)")
    ap.add_argument("--reps", type=int, default=3, help="calls timed by --micro")
    args = ap.parse_args()
    tpg = args.tokens
    if args.micro:
        device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(device)
        micro.tokens = tpg
        micro(args.micro, device, args.reps)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            # each step: one bounded sample (args.cpu_tokens tokens) of the workload
            cb = cpu_reference_ffn(args.cpu_tokens, D_MODEL, D_FF, args.steps, args.warmup,
                                   sparsity=SPARSITY)
            line = {"impl": "reference", "metric": METRIC, "value": cb["value"],
                    "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
                    "warmup": args.warmup, "higher_is_better": True, "dtype": "f32",
                    "data": "synthetic (seeded)",
                    "config": workload_config(tpg, world, tpg * world),
                    "cpu_baseline": cb,
                    "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                            "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
        return

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    import autoresearch2_b200 as _sf
    _sf.set_sparse_mma(args.sparse_mma)
    if args.pack_only:
        pk = peaks()
        for p in PACK_SWEEP:
            r = bench_pack(device, p)
            r["pack_frac"] = round(r["pack_gbs"] / pk["hbm_gbs"], 3)
            r["unpack_frac"] = round(r["unpack_gbs"] / pk["hbm_gbs"], 3)
            print(json.dumps(r), flush=True)
            torch.cuda.empty_cache()
        return
    group = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
        group = dist.group.WORLD
    torch.backends.cuda.matmul.allow_tf32 = False

    x, W1, W2, b1, dout = make_ffn_inputs(tpg, D_MODEL, D_FF, SPARSITY, device, seed=rank)
    step = Step(x, W1, W2, b1, dout, group)
    step()
    torch.cuda.synchronize(device)
    s_meas = 1.0 - step.buf.used() / (tpg * D_FF)

    import autoresearch2_b200 as sf
    from autoresearch2_b200 import _lib
    sf.check_status(device)
    n0 = _lib.launch_count
    step()
    launches_per_step = _lib.launch_count - n0
    with ClockSampler(local) as clk, _lib.KernelTimer() as ktimer:
        ms = time_steps(step, args.steps, args.warmup, device)
    clocks = clk.summary()
    # a bounded device wait that ran out inside the timed steps would show here
    status_after = sf.check_status(device, raise_on_error=False)
    tokens = tpg * world
    value = tokens / (ms / 1e3)
    kernels = kernel_breakdown(ktimer, args.steps + args.warmup, ms)

    # end to end: every step copies that step's inputs -- the activations x and
    # the upstream gradient dout -- from pinned host memory and reads its loss
    # back.  As a training loop's input pipeline would, the copies of the next
    # step's inputs run on a second stream into the other of two device buffer
    # pairs while this step computes (PCIe and the SMs work side by side); each
    # step waits for its own inputs' copies.
    x_host = x.cpu().pin_memory()
    dout_host = dout.cpu().pin_memory()
    copy_stream = torch.cuda.Stream(device)
    bufs = [(torch.empty_like(x), torch.empty_like(dout)) for _ in range(2)]
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    free = [torch.cuda.Event(), torch.cuda.Event()]
    pipe = {"i": 0, "primed": False}

    def issue_copy(k):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[k])  # the buffers' previous step is done with them
            bufs[k][0].copy_(x_host, non_blocking=True)
            bufs[k][1].copy_(dout_host, non_blocking=True)
            ready[k].record(copy_stream)

    loss_holder = {}

    def e2e_step():
        k = pipe["i"] % 2
        if not pipe["primed"]:
            issue_copy(k)
            pipe["primed"] = True
        torch.cuda.current_stream(device).wait_event(ready[k])
        issue_copy(1 - k)  # the next step's inputs, during this step
        out = step(*bufs[k])
        free[k].record(torch.cuda.current_stream(device))
        loss_holder["l"] = float(out.float().pow(2).mean().item())
        pipe["i"] += 1

    e2e = None
    if not args.quick:
        e2e_ms = time_steps(e2e_step, max(3, args.steps // 2), 3, device)
        e2e = {"value": round(tokens / (e2e_ms / 1e3), 1), "unit": "tokens/s",
               "h2d_bytes_per_step": x.numel() * x.element_size() + dout.numel() * dout.element_size(),
               "d2h_bytes_per_step": 4}

    extras = {}
    if rank == 0 and not args.quick:
        dense = DenseStep(x, W1, W2, b1, dout)
        d_ms = time_steps(dense, args.steps, args.warmup, device) if world == 1 else None
        if d_ms is not None:
            extras["dense_cublas"] = {"tokens_per_s": round(tpg / (d_ms / 1e3), 1),
                                      "ms_per_step": round(d_ms, 3)}
            extras["speedup_vs_dense"] = round(d_ms / ms, 3)
        del dense
    if world == 1 and not args.no_sweep and not args.quick:
        sweep = {}
        for s in SWEEP:
            xs, W1s, W2s, b1s, dos = make_ffn_inputs(tpg, D_MODEL, D_FF, s, device)
            st = Step(xs, W1s, W2s, b1s, dos)
            k = max(3, args.steps // 2)
            # 4 warm-up steps: the auto mode reads the sparsity the first step observed
            sm = time_steps(st, k, 4, device)
            used = st.buf.used()
            forced = {}
            for mode in ("off", "on"):  # the two product paths the auto mode chooses between
                sf.set_sparse_mma(mode)
                forced[mode] = time_steps(st, k, 2, device)
            sf.set_sparse_mma(args.sparse_mma)
            dm = time_steps(DenseStep(xs, W1s, W2s, b1s, dos), k, 2, device)
            sweep[str(s)] = {"tokens_per_s": round(tpg / (sm / 1e3), 1),
                             "dense_products_tokens_per_s": round(tpg / (forced["off"] / 1e3), 1),
                             "sp24_products_tokens_per_s": round(tpg / (forced["on"] / 1e3), 1),
                             "dense_tokens_per_s": round(tpg / (dm / 1e3), 1),
                             "measured_sparsity": round(1.0 - used / (tpg * D_FF), 4)}
            del st, xs, W1s, W2s, b1s, dos
            torch.cuda.empty_cache()
        extras["sweep"] = sweep

    pk = peaks()
    roof = roofline(kernels, tpg, pk, s_meas)
    clustered = None
    if not args.quick and not args.no_clustered:
        # every rank runs it (its weight gradients are all-reduced)
        clustered = bench_clustered(device, group, world, max(3, args.steps // 4), args.warmup, pk, rank)
    flops = step_flops(step, ms, s_meas, pk) if rank == 0 else None
    pack = codec = deep_ffn = gpt_step = None
    if not args.quick and world > 1:
        # the GPT harness data-parallel on every rank (its gradients all-reduced)
        gpt_step = bench_gpt(device, peaks(), world=world, rank=rank)
    if rank == 0 and not args.quick:
        pack = bench_pack(device)
        pack["pack_frac_of_measured_hbm"] = round(pack["pack_gbs"] / pk["hbm_gbs"], 3)
        pack["unpack_frac_of_measured_hbm"] = round(pack["unpack_gbs"] / pk["hbm_gbs"], 3)
        sweep_p = {}
        for p in PACK_SWEEP:
            if p != PACK_P:
                r = bench_pack(device, p, reps=10)
                sweep_p[str(p)] = {"pack_gbs": r["pack_gbs"], "unpack_gbs": r["unpack_gbs"]}
        pack["sweep_p"] = sweep_p
        codec = bench_codec15(device)
        if world == 1:  # single-GPU harnesses; at N > 1 the other ranks would wait on them
            deep_ffn = bench_deep(device)
            gpt_step = bench_gpt(device, peaks())
        for k in ("compress", "uncompress"):
            codec[f"{k}_frac_of_measured_hbm"] = round(codec[f"{k}_gbs"] / pk["hbm_gbs"], 3)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded; inputs larger than L2, no flush)",
            "config": workload_config(tpg, world, tokens, s_meas), "sparse_mma": args.sparse_mma,
            "e2e": e2e, "clocks": clocks, "roofline": roof, "kernels": kernels, "pack": pack,
            "codec15": codec, "deep_ffn": deep_ffn, "gpt": gpt_step, "flops": flops,
            "gpu_launches": launches_per_step * args.steps,
            "device_status_after_timed": status_after, "clustered": clustered,
        }
        line.update(extras)
        if world == 1 and not args.quick:
            try:
                # about 10 s of host work: 8 samples after one untimed
                line["cpu_baseline"] = cpu_baselines(args.cpu_tokens, steps=6, warmup=1)
            except Exception as e:  # noqa: BLE001
                line["cpu_baseline"] = {"error": repr(e)}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if status_after:
        sys.exit(f"device status 0x{status_after:x} after the timed steps: the run is not valid")


if __name__ == "__main__":
    main()
