"""Denoising-transformer training, data-parallel with one process per GPU.

Model: the reference's denoise layer (tests/main_denoise.py:11-54) - pre-LN
self-attention with a residual add, pre-LN feed-forward (Linear, ReLU, Linear)
with a residual add, then a final LayerNorm - stacked `layers` deep and built
from the PureAttention operators; MSE loss against the clean signal and Adam
(src/core/Adam.cpp:28-59), as the reference's training loop does
(tests/main_denoise.py:79-110).

Data: each sequence is a sum of four sinusoids a*sin(f*t + phi), f ~ U(0.5, 8),
phi ~ U(0, 2pi), a ~ U(0.2, 1), sampled at `seq` points of t in [0, 1); a fixed
Linear(1 -> embed) map (weights and bias U(-1, 1), the same on every rank)
lifts it to [batch, seq, embed]. The input adds N(0, noise^2) to that lift and
the target is the clean lift, so output and target have the reference's
[batch, seq, embed] shape (tests/main_denoise.py:69-77).

Data parallelism: every rank builds the model from the same seed and rank 0's
parameters are broadcast once, so all replicas start identical. Each rank runs
forward and backward on its own sequences; `GradAllReduce` then averages the
weight gradients over ranks with NCCL all-reduce, in buckets: the parameters'
gradients are moved into one flat arena per bucket, so each bucket is one
in-place all-reduce, started as soon as backward has finished its gradients;
every rank then takes the same Adam step.

Precision: weights, activations and gradients are fp32 tensors. math="split3"
computes every product at fp32-level accuracy (bf16 hi/lo planes, three
products); math="bf16" rounds the operands of each matmul and attention to
bf16 (one product, fp32 accumulation) - mixed-precision training with fp32
master weights and fp32 Adam.

Stream order: the operators run on the CUDA legacy default stream, which is
also torch's default stream, so the torch copies and process-group collectives
issued from the same thread are ordered with them without host syncs.

CUDA graph (graph=True, the default; with a gradient all-reduce its
overlapped NCCL buckets are captured with the backward): the first step on an input
buffer captures zero_grad, forward, MSE and backward - about 340 kernel
launches, the stream-ordered allocations and frees of the step's activations
and the loss copied into a persistent scalar - into a CUDA graph on a side
stream; later steps replay it and run Adam after it. Replay removes the host
work and the launch gaps between the kernels. The side stream waits for the
default stream before each step and the default stream for it after, so
callers see the same order as eager steps. A graph is kept per input buffer
and f32 math mode (the mode is fixed at capture).
"""
import math

import numpy as np

import PureAttention as pa


class FeedForward(pa.Module):
    """Linear(embed, hidden) -> ReLU -> Linear(hidden, embed)
    (tests/main_denoise.py:11-25). fused=True runs the first Linear and the
    ReLU as one op (the clamp in the GEMM epilogue, the mask folded into its
    backward); the parameters are the same either way."""

    def __init__(self, embed_dim, hidden_dim, fused=True):
        super().__init__()
        self.fc1 = pa.Linear(embed_dim, hidden_dim, relu=fused)
        self.relu = None if fused else pa.ReLU()
        self.fc2 = pa.Linear(hidden_dim, embed_dim)

    def forward(self, x):
        h = self.fc1.forward(x)
        if self.relu is not None:
            h = self.relu.forward(h)
        return self.fc2.forward(h)

    def parameters(self):
        return self.fc1.parameters() + self.fc2.parameters()


class TransformerLayer(pa.Module):
    """Pre-LN attention and feed-forward sublayers with residual adds and a
    final LayerNorm (tests/main_denoise.py:27-54)."""

    def __init__(self, embed_dim, num_heads, ffn_dim):
        super().__init__()
        self.mha = pa.MultiheadAttention(embed_dim, num_heads)
        self.ln1 = pa.LayerNorm(embed_dim)
        self.ffn = FeedForward(embed_dim, ffn_dim)
        self.ln2 = pa.LayerNorm(embed_dim)
        self.ln_final = pa.LayerNorm(embed_dim)

    def forward(self, x):
        x_norm = self.ln1.forward(x)
        # each residual add is fused with the LayerNorm that reads its sum
        x, h = self.ln2.forward_add(x, self.mha.forward(x_norm, x_norm, x_norm))
        _, out = self.ln_final.forward_add(x, self.ffn.forward(h))
        return out

    def parameters(self):
        return (self.mha.parameters() + self.ln1.parameters() + self.ffn.parameters()
                + self.ln2.parameters() + self.ln_final.parameters())


class DenoiseTransformer(pa.Module):
    def __init__(self, layers, embed_dim, num_heads, ffn_dim):
        super().__init__()
        self.layers = [TransformerLayer(embed_dim, num_heads, ffn_dim) for _ in range(layers)]

    def forward(self, x):
        for layer in self.layers:
            x = layer.forward(x)
        return x

    def parameters(self):
        return [p for layer in self.layers for p in layer.parameters()]


def embedding(embed, seed):
    """The fixed Linear(1 -> embed) lift: (weight, bias), U(-1, 1) each."""
    rng = np.random.default_rng(seed)
    return (rng.uniform(-1.0, 1.0, embed).astype(np.float32),
            rng.uniform(-1.0, 1.0, embed).astype(np.float32))


def denoise_batch(rng, batch, seq, lift, noise=0.1):
    """(noisy input, clean target), float32 [batch, seq, embed] each."""
    t = np.arange(seq, dtype=np.float64) / seq
    f = rng.uniform(0.5, 8.0, (batch, 4, 1))
    phi = rng.uniform(0.0, 2.0 * math.pi, (batch, 4, 1))
    a = rng.uniform(0.2, 1.0, (batch, 4, 1))
    signal = (a * np.sin(f * t + phi)).sum(axis=1)                  # [batch, seq]
    w, b = lift
    clean = (signal[..., None] * w + b).astype(np.float32)          # [batch, seq, embed]
    noisy = clean + rng.normal(0.0, noise, clean.shape).astype(np.float32)
    return noisy, clean


def _torch():
    import torch
    return torch


def device_view(t):
    """torch view (no copy) of a PureAttention tensor's data."""
    return _torch().as_tensor(t, device="cuda")


def grad_view(t):
    """torch view (no copy) of a PureAttention tensor's gradient."""
    return _torch().as_tensor(t.grad_view(), device="cuda")


def plan_buckets(nbytes, bucket_bytes, tail_bytes=0, tail_bucket_bytes=None):
    """Buckets (lists of indices into nbytes) in reverse index order - the
    order in which backward finishes the gradients. Each bucket holds at most
    bucket_bytes (a gradient larger than that gets a bucket of its own); the
    last tail_bytes of that order (the gradients backward finishes last, whose
    reduction cannot hide behind it) go into buckets of tail_bucket_bytes."""
    order = list(range(len(nbytes)))[::-1]
    total = sum(nbytes)
    buckets, cur, cur_bytes, seen = [], [], 0, 0
    for i in order:
        limit = bucket_bytes
        if tail_bucket_bytes and seen >= total - tail_bytes:
            limit = tail_bucket_bytes
        if cur and cur_bytes + nbytes[i] > limit:
            buckets.append(cur)
            cur, cur_bytes = [], 0
        cur.append(i)
        cur_bytes += nbytes[i]
        seen += nbytes[i]
    if cur:
        buckets.append(cur)
    return buckets


class GradAllReduce:
    """Average gradients over the ranks of a process group, in buckets.

    `grads` are flat-viewable torch tensors (views of the gradient buffers),
    packed into buckets by plan_buckets. By default each bucket owns a flat
    buffer; a call gathers the bucket into it, all-reduces it and scatters the
    averaged values back. for_tensors() instead moves the gradients of
    PureAttention tensors into one flat arena per bucket, so the all-reduce
    runs in place with no gather or scatter. NCCL averages in the collective
    (ReduceOp.AVG); other backends sum and then divide by the world size.

    Overlapped use: begin(), then ready(key) for each gradient once it is
    final (keys[i] names grads[i]; by default its data pointer), then
    finish(). A bucket is reduced as soon as all of its gradients are ready,
    buckets strictly in index order so that every rank issues the same
    collectives in the same order; CUDA buckets run on a side stream that
    waits for the point in the default stream where the bucket became ready,
    and finish() makes the default stream wait for them.
    """

    def __init__(self, grads, bucket_bytes=100 << 20, group=None, keys=None, tail_bytes=0,
                 tail_bucket_bytes=None, arenas=None, plan=None):
        torch = _torch()
        import torch.distributed as dist
        self.dist, self.group = dist, group
        self.world = dist.get_world_size(group)
        self.avg_in_collective = dist.get_backend(group) == "nccl"
        grads = list(grads)
        if plan is None:
            plan = plan_buckets([g.numel() * g.element_size() for g in grads], bucket_bytes,
                                tail_bytes, tail_bucket_bytes)
        self.plan = plan
        self.buckets = [[grads[i].view(-1) for i in b] for b in plan]
        self.inplace = arenas is not None  # the views already are slices of the arenas
        self.flat = (list(arenas) if self.inplace else
                     [torch.empty(sum(v.numel() for v in b), dtype=b[0].dtype, device=b[0].device)
                      for b in self.buckets])
        self.sizes = [[v.numel() for v in b] for b in self.buckets]
        keys = [g.data_ptr() for g in grads] if keys is None else list(keys)
        if len(keys) != len(grads):
            raise ValueError("one key per gradient")
        self.where = {keys[i]: b for b, idx in enumerate(plan) for i in idx}
        cuda = grads[0].device.type == "cuda"
        self.comm = torch.cuda.Stream(device=grads[0].device) if cuda else None
        self.pending = None

    @classmethod
    def for_tensors(cls, tensors, bucket_bytes=100 << 20, group=None, tail_bytes=0,
                    tail_bucket_bytes=None):
        """Reducer over the gradients of PureAttention tensors, which are moved
        (Tensor.set_grad_storage, zeroed) into one flat arena per bucket: each
        gradient's slot starts on a 256-byte boundary, and the bucket's
        all-reduce runs on its arena in place. The reducer owns the arenas and
        must outlive the tensors' use of their gradients."""
        torch = _torch()
        numel = [int(np.prod(t.shape())) for t in tensors]
        plan = plan_buckets([4 * n for n in numel], bucket_bytes, tail_bytes, tail_bucket_bytes)
        pad = lambda n: (n + 63) // 64 * 64  # floats: 256-byte slots
        arenas, views = [], [None] * len(tensors)
        for idx in plan:
            arena = torch.zeros(sum(pad(numel[i]) for i in idx), dtype=torch.float32, device="cuda")
            off = 0
            for i in idx:
                tensors[i].set_grad_storage(arena.data_ptr() + 4 * off)
                views[i] = arena[off:off + numel[i]]
                off += pad(numel[i])
            # the arena is reduced whole: padding stays zero on every rank
            arenas.append(arena)
        torch.cuda.synchronize()  # the rebinds' memsets ran on the operators' stream
        return cls(views, group=group, arenas=arenas, plan=plan)

    def _reduce(self, b):
        torch = _torch()
        op = self.dist.ReduceOp.AVG if self.avg_in_collective else self.dist.ReduceOp.SUM
        views, flat, sizes = self.buckets[b], self.flat[b], self.sizes[b]
        if not self.inplace:
            torch.cat(views, out=flat)
        self.dist.all_reduce(flat, op=op, group=self.group)
        if not self.avg_in_collective:
            flat.div_(self.world)
        if not self.inplace:
            torch._foreach_copy_(views, list(torch.split(flat, sizes)))

    def __call__(self):
        for b in range(len(self.buckets)):
            self._reduce(b)

    def begin(self):
        self.pending = [len(v) for v in self.buckets]
        self.launched = 0  # buckets 0 .. launched-1 are reduced or queued

    def _launch(self, b):
        if self.comm is None:
            self._reduce(b)
            return
        torch = _torch()
        ready = torch.cuda.Event()
        ready.record()  # the current stream, where this bucket's gradients were written
        with torch.cuda.stream(self.comm):
            self.comm.wait_event(ready)
            self._reduce(b)

    def ready(self, key):
        b = self.where.get(key)
        if b is None or self.pending is None:
            return
        self.pending[b] -= 1
        while self.launched < len(self.buckets) and self.pending[self.launched] == 0:
            self._launch(self.launched)
            self.launched += 1

    def finish(self):
        """Reduce the buckets not reduced yet (gradients no node wrote) and
        make the current stream wait for every reduction."""
        while self.launched < len(self.buckets):
            self._launch(self.launched)
            self.launched += 1
        self.pending = None
        if self.comm is not None:
            _torch().cuda.current_stream().wait_stream(self.comm)

    @property
    def nbytes(self):
        return sum(f.numel() * f.element_size() for f in self.flat)


class DenoiseTrainer:
    """One replica of the data-parallel denoise training loop.

    step(x, t) takes one batch from (pinned) host memory: copies it to the
    device, runs forward, MSE, backward, the gradient all-reduce (when a
    process group with more than one rank is up) and Adam, and returns the
    loss as a float. step_resident() runs the same step on the batch already
    on the device and returns the loss tensor without a host read.
    """

    def __init__(self, layers=6, embed=1024, heads=16, ffn=4096, seq=2048, batch=8, lr=1e-4,
                 seed=5, bucket_bytes=100 << 20, group=None, math="split3", tail_bytes=0,
                 tail_bucket_bytes=None, graph=None):
        import torch.distributed as dist
        self.shape = (batch, seq, embed)
        self.math = math
        pa.set_float32_math(math)  # fp32 master weights; "bf16": bf16 products
        pa.set_seed(seed)  # same initial weights on every rank
        self.model = DenoiseTransformer(layers, embed, heads, ffn)
        self.params = self.model.parameters()
        self.opt = pa.Adam(self.params, lr=lr)
        self.criterion = pa.MSE()
        self.x = pa.Tensor(list(self.shape), False)
        self.t = pa.Tensor(list(self.shape), False)
        self.x_dev, self.t_dev = device_view(self.x), device_view(self.t)
        self.reducer = None
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            src = dist.get_global_rank(group, 0) if group is not None else 0
            for p in self.params:
                dist.broadcast(device_view(p), src=src, group=group)
            # gradients live in per-bucket arenas: each bucket is all-reduced in place
            self.reducer = GradAllReduce.for_tensors(self.params, bucket_bytes, group, tail_bytes,
                                                     tail_bucket_bytes)
        self.overlap = True  # all-reduce each bucket while the rest of the backward runs
        # replay the forward + backward as a CUDA graph (with a gradient
        # all-reduce, its overlapped NCCL buckets are captured with the backward)
        self.graph = True if graph is None else bool(graph)
        self._graphs = {}  # (input tensor, math) -> torch.cuda.CUDAGraph
        self._gstream = None
        self._loss = None

    def _leaf_ready(self, t):
        self.reducer.ready(t.grad_view().__cuda_array_interface__["data"][0])

    @property
    def num_parameters(self):
        return sum(int(np.prod(p.shape())) for p in self.params)

    def load(self, x_host, t_host):
        """Queue the copies of one batch (torch CPU tensors, pinned for
        asynchronous copies) into the input tensors."""
        self.x_dev.view(x_host.shape).copy_(x_host, non_blocking=True)
        self.t_dev.view(t_host.shape).copy_(t_host, non_blocking=True)

    def _forward_backward(self):
        """zero_grad, forward, MSE, backward into self._loss (graph capture body:
        every tensor of the step is freed before it returns)."""
        import pa_capi
        self.opt.zero_grad()
        out = self.model.forward(self.x)
        loss = self.criterion(out, self.t)
        if self.reducer is not None:
            self.reducer.begin()
            loss.backward(True, self._leaf_ready)
            self.reducer.finish()
        else:
            loss.backward()
        lib, st = pa_capi.load(), pa.get_stream()
        dst = self._loss.__cuda_array_interface__["data"][0]
        if (lib.pa_fill(dst, 1, 0.0, st) != 0 or
                lib.pa_grad_accumulate(loss.__cuda_array_interface__["data"][0], dst, 1, st) != 0):
            raise RuntimeError("DenoiseTrainer: loss copy failed")
        del out, loss

    def _step_graph(self):
        torch = _torch()
        if self._gstream is None:
            self._gstream = torch.cuda.Stream()
            self._loss = pa.Tensor([1], False)
        main, s = torch.cuda.current_stream(), self._gstream
        prev = pa.get_stream()
        s.wait_stream(main)  # inputs and earlier steps first
        pa.set_stream(s.cuda_stream)
        try:
            key = (id(self.x), self.math)
            g = self._graphs.get(key)
            with torch.cuda.stream(s):
                if g is None:
                    for k in [k for k in self._graphs if k[0] == key[0]]:
                        del self._graphs[k]  # a graph of the same input in another math mode
                    self._forward_backward()  # eager once: first-use setup outside the capture
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=s):
                        self._forward_backward()
                    self._graphs[key] = g
                g.replay()
                self.opt.step()
        finally:
            pa.set_stream(prev)
        main.wait_stream(s)
        return self._loss

    def release_graphs(self):
        """Drop the captured graphs (before destroying a process group whose
        collectives they hold)."""
        self._graphs.clear()

    def step_resident(self):
        pa.set_float32_math(self.math)
        if self.graph:
            return self._step_graph()
        self.opt.zero_grad()
        out = self.model.forward(self.x)
        loss = self.criterion(out, self.t)
        if self.reducer is not None and self.overlap:
            self.reducer.begin()
            loss.backward(True, self._leaf_ready)
            self.reducer.finish()
        else:
            loss.backward()
            if self.reducer is not None:
                self.reducer()
        del out
        self.opt.step()
        return loss  # holds this step's graph until the caller drops it

    def step(self, x_host, t_host):
        self.load(x_host, t_host)
        return float(device_view(self.step_resident()).item())

    def train(self, batches):
        """Pipelined loop over (x, t) batches in pinned host memory; returns
        the losses. Batch i+1 is copied on a side stream into the second
        input buffer while step i computes, and each step's loss is copied to
        pinned host memory without blocking and read one step later, so the
        host keeps the GPU fed (what step() cannot do: it copies, then waits
        for the loss)."""
        torch = _torch()
        batches = list(batches)
        if not batches:
            return []
        if not hasattr(self, "_bufs"):
            self._bufs = [(self.x, self.t)] + [
                (pa.Tensor(list(self.shape), False), pa.Tensor(list(self.shape), False))]
            self._copy_stream = torch.cuda.Stream()
            self._loss_host = torch.empty(2, dtype=torch.float32).pin_memory()
        main = torch.cuda.default_stream()  # the operators' stream
        cs = self._copy_stream
        copied = [torch.cuda.Event() for _ in range(2)]
        freed = [torch.cuda.Event() for _ in range(2)]
        read = [torch.cuda.Event() for _ in range(2)]

        def copy_in(i):
            x, t = batches[i]
            bx, bt = self._bufs[i % 2]
            with torch.cuda.stream(cs):
                if i >= 2:
                    cs.wait_event(freed[i % 2])  # step i-2 is done with this buffer
                device_view(bx).view(x.shape).copy_(x, non_blocking=True)
                device_view(bt).view(t.shape).copy_(t, non_blocking=True)
                copied[i % 2].record(cs)

        losses = []
        copy_in(0)
        for i in range(len(batches)):
            if i + 1 < len(batches):
                copy_in(i + 1)
            main.wait_event(copied[i % 2])
            self.x, self.t = self._bufs[i % 2]
            loss = self.step_resident()
            freed[i % 2].record(main)
            if i >= 2:
                read[i % 2].synchronize()  # loss of step i-2 (its slot is reused now)
                losses.append(float(self._loss_host[i % 2]))
            self._loss_host[i % 2].copy_(device_view(loss).view(()), non_blocking=True)
            read[i % 2].record(main)
            del loss
        for i in range(max(0, len(batches) - 2), len(batches)):
            read[i % 2].synchronize()
            losses.append(float(self._loss_host[i % 2]))
        self.x, self.t = self._bufs[0]
        return losses

    def save(self, path):
        """Parameters, Adam moments and step count to an .npz file."""
        m, v = self.opt.state()
        arrays = {}
        for i, p in enumerate(self.params):
            arrays["p%d" % i] = device_view(p).cpu().numpy()
            arrays["m%d" % i] = device_view(m[i]).cpu().numpy()
            arrays["v%d" % i] = device_view(v[i]).cpu().numpy()
        np.savez(path, step=np.int64(self.opt.step_count), **arrays)

    def restore(self, path):
        torch = _torch()
        m, v = self.opt.state()
        with np.load(path) as z:
            if sum(1 for k in z.files if k.startswith("p")) != len(self.params):
                raise ValueError("checkpoint holds a different number of parameters")
            for i, p in enumerate(self.params):
                for name, t in (("p", p), ("m", m[i]), ("v", v[i])):
                    a = z["%s%d" % (name, i)]
                    if list(a.shape) != list(t.shape()):
                        raise ValueError("checkpoint shape mismatch at %s%d" % (name, i))
                    device_view(t).copy_(torch.from_numpy(a))
            self.opt.step_count = int(z["step"])
