"""Linear/MLP training on the B200 matmul path, data-parallel across GPUs.

This mirrors one training step of the reference (``Experiment::train_step``,
moonxi-net/train/train.mbt:40-54, driven by ``run_gpu``,
moonxi-net-gpu/train/run.mbt:41-57) for a stack of Linear layers with ReLU
between them, cross-entropy with integer labels and momentum SGD with
global-norm clipping.  The arithmetic follows the reference's autograd tape:

* forward per layer ``x.matmul(w).add(b)`` then ``relu`` (layers.mbt:59-64;
  layout "nn", w stored [in, out]) or ``x.matmul(w.transpose())``
  (mlp.mbt:16-23; layout "nt", w stored [out, in]) -- one fused
  ``moonbit_cuda_linear_fwd`` call (GEMM + broadcast bias + ReLU epilogue);
* backward closures of grad/blas.mbt:23-39 (dW = X^T dY, dX = dY W^T, run as
  TN / NT GEMMs on the stored operands, no transpose materialised),
  grad/grad.mbt:163-174 (db = column sum) and grad/image.mbt:45-61 (ReLU
  mask); the first layer's dX is skipped because the input has no gradient
  (grad/grad.mbt:80-85);
* update: momentum SGD with auto clipping (nparray/trait_impl.mbt:280-311)
  over one flat parameter buffer, on the device, with no host round trip.

Data parallelism (new; the reference has none): the batch is split by rows
over the ranks of a ``torch.distributed`` process group; the loss is scaled by
1/global_batch so the sum over ranks equals the single-device mean; each
layer's (dW, db) bucket is all-reduced (NCCL over NVLink) as soon as its
GEMMs are queued, so the reduction of layer i overlaps the backward GEMMs of
layers i-1..1; every replica then applies the identical update.  On an NCCL
group the collectives go through the library's own ``moonbit_nccl_*`` stubs
(collectives.NcclCollectives; torch.distributed only bootstraps the
communicator), on a gloo group through torch.distributed.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops
from .collectives import as_collectives

_ALIGN = 64  # floats: every parameter block starts on a 256-byte boundary
_LOSS_SLOTS = _ALIGN  # the per-step loss rides in front of the first bucket


def _round_up(x: int, a: int = _ALIGN) -> int:
    return (x + a - 1) // a * a


class FlatLayout:
    """Offsets of the flat parameter / gradient / velocity buffers.

    Parameters follow the reference's order [w1, b1, w2, b2, ...]
    (MLP::params, moonxi-net/model/mlp.mbt:27-29); each block starts on a
    256-byte boundary (zero padding between blocks).  The gradient buffer is
    prefixed by a 64-float slot that carries the step's loss, so that the
    loss rides in the first layer's all-reduce bucket.  With shard_world = G
    > 1 every bucket is padded (zeros after its bias) to a multiple of G x 64
    floats, so it splits into G equal 256-byte aligned pieces (ShardPlan).
    Device-independent: the data-parallel host logic is tested with it on CPU
    ranks.
    """

    def __init__(self, dims, shard_world: int = 1):
        self.dims = list(dims)
        self.L = len(dims) - 1
        self.shard_world = int(shard_world)
        self.w_off, self.b_off = [], []
        # offsets in gradient-buffer coordinates (loss slot first), then shifted
        cur = _LOSS_SLOTS
        for i in range(self.L):
            fi, fo = self.dims[i], self.dims[i + 1]
            self.w_off.append(cur - _LOSS_SLOTS)
            cur += _round_up(fi * fo)
            self.b_off.append(cur - _LOSS_SLOTS)
            cur += _round_up(fo)
            cur = _round_up(cur, _ALIGN * self.shard_world)  # bucket boundary
        self.n_flat = cur - _LOSS_SLOTS
        self.grads_buf_len = cur

    def w_range(self, i):
        return self.w_off[i], self.w_off[i] + self.dims[i] * self.dims[i + 1]

    def b_range(self, i):
        return self.b_off[i], self.b_off[i] + self.dims[i + 1]

    def bucket(self, i):
        """[start, end) in the gradient buffer of layer i's all-reduce bucket
        (its dW and db; bucket 0 also holds the loss slot)."""
        start = self.w_off[i] + _LOSS_SLOTS if i > 0 else 0
        end = _LOSS_SLOTS + (self.w_off[i + 1] if i + 1 < self.L else self.n_flat)
        return start, end

    def reduce_order(self):
        """Buckets in the order backward produces them (last layer first)."""
        return list(reversed(range(self.L)))


class ShardPlan:
    """Partition of the flat buffers for a data-parallel update sharded over
    `world` ranks.  Coordinates are those of the gradient buffer (the loss
    slot first); the parameter, velocity and split-copy buffers carry the same
    front slot so one range means the same parameters in all of them.  Each
    layer's bucket splits into `world` equal contiguous pieces; rank r
    reduce-scatters into, owns and updates piece r of every bucket, and
    all-gathers the others' pieces of the new weights.  The reduce-scatter
    and the all-gather are in place (the rank's piece is a view of the
    bucket), which NCCL and gloo both accept."""

    def __init__(self, layout: FlatLayout, world: int, rank: int):
        if layout.shard_world != world:
            raise ValueError("layout was not padded for this world size")
        self.layout, self.world, self.rank = layout, world, rank
        self.buckets = [layout.bucket(i) for i in range(layout.L)]
        self.pieces = []
        for s, e in self.buckets:
            per = (e - s) // world
            assert per * world == e - s and per % _ALIGN == 0
            self.pieces.append((s + rank * per, s + (rank + 1) * per))

    def update_ranges(self):
        """This rank's parameter ranges (its pieces minus the loss slot)."""
        out = []
        for a, b in self.pieces:
            a = max(a, _LOSS_SLOTS)
            if b > a:
                out.append((a, b))
        return out

    def reduce_scatter(self, buf, i, group, async_op=True, overlap=True):
        """Sums bucket i of `buf` over the ranks into this rank's piece.
        `group`: a process group (None = default) or a collectives object;
        overlap=False: nothing runs beside it (it may take every SM)."""
        s, e = self.buckets[i]
        a, b = self.pieces[i]
        return as_collectives(group).reduce_scatter(buf[a:b], buf[s:e], async_op=async_op,
                                                    overlap=overlap)

    def all_gather(self, buf, i, group, async_op=True, overlap=True):
        """Fills bucket i of `buf` with every rank's piece."""
        s, e = self.buckets[i]
        a, b = self.pieces[i]
        return as_collectives(group).all_gather(buf[s:e], buf[a:b], async_op=async_op,
                                                overlap=overlap)


def shard_rows(global_batch: int, rank: int, world: int):
    """[begin, end) of this rank's rows of the global batch (equal shards)."""
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} not divisible by {world} ranks")
    per = global_batch // world
    return rank * per, (rank + 1) * per


class MLP:
    """A stack of Linear layers (ReLU between them) trained with momentum SGD.

    Parameters live in one flat device buffer in the reference's parameter
    order [w1, b1, w2, b2, ...]; gradients and velocities use the same layout.
    """

    def __init__(self, dims, weights=None, biases=None, layout: str = "nn", device=None,
                 precision="default", lr: float = 0.01, momentum: float = 0.9,
                 weight_decay: float = 1e-4, max_grad_norm: float = 35.0,
                 process_group=None, fused=None, shard_update=None, collectives=None,
                 pair_backward=None):
        if layout not in ("nn", "nt"):
            raise ValueError("layout must be 'nn' (w [in,out]) or 'nt' (w [out,in])")
        self.dims = list(dims)
        self.L = len(dims) - 1
        self.layout = layout
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        # The model's library context carries the precision mode, so the
        # adjacent ops follow it too ("nparray": NpArray operation order).
        self.precision = precision
        # the model's own context: its workspace, status word and SM budget
        self.ctx = ops.new_context(self.device.index, precision)
        self.lr, self.momentum = float(lr), float(momentum)
        self.weight_decay, self.max_grad_norm = float(weight_decay), float(max_grad_norm)
        self.pg = process_group
        self.rank = 0
        # collectives: None = the group's default (the library's NCCL stubs on
        # an NCCL group, torch.distributed otherwise), "torch" = always
        # torch.distributed, or a collectives object to share
        self.coll = None
        # SMs left to the collectives that overlap the GEMMs (a persistent GEMM
        # CTA and an NCCL CTA do not fit on one SM together): the GEMMs prefer
        # the rest (on 148 SMs the 128 left also make every power-of-two tile
        # count a whole number of waves) and each NCCL collective is capped to
        # them, so that all its channels run at once beside a GEMM
        import os
        self.comm_sms = int(os.environ.get("MX_COMM_SMS", "20"))
        if process_group is not None:
            import torch.distributed as dist
            self.world = dist.get_world_size(process_group)
            self.rank = dist.get_rank(process_group)
            if collectives == "torch":
                from .collectives import TorchCollectives
                self.coll = TorchCollectives(process_group)
            elif collectives is not None:
                self.coll = collectives
            else:
                self.coll = as_collectives(process_group, self.device,
                                           max_ctas=self.comm_sms if self.world > 1 else 0)
        else:
            self.world = 1
        self._owns_coll = collectives is None and self.coll is not None
        if self.world > 1:
            sms = torch.cuda.get_device_properties(self.device).multi_processor_count
            ops.set_sm_budget(self.ctx, sms - self.comm_sms)
        # Split-form path (3xTF32 with every operand kept as hi/lo copies written
        # by its producer): needs TMA-legal leading dimensions (multiples of 4).
        self.fused = (precision == "3xtf32" and all(d % 4 == 0 for d in self.dims)
                      and fused is not False)
        # Sharded update (split-form path, several ranks): gradients are
        # reduce-scattered instead of all-reduced, each rank updates its 1/G
        # of the parameters, and the new weights are all-gathered layer by
        # layer (the first at the end of the step, the others beside the next
        # step's forward), where each rank re-splits them.  Default from 4
        # ranks on: measured on B200s (wide MLP, global batch 8192) it gives
        # 2.63 vs 2.40 M samples/s on 4 GPUs and 3.73 vs 3.42 M on 8, while
        # on 2 the replicated update is ahead (1.47 vs 1.39 M: the update is
        # only halved there, and the gathers cost the forward more).
        if shard_update is None:
            shard_update = self.world >= 4
        self.sharded = self.fused and self.world > 1 and bool(shard_update)
        if self.sharded:
            # the weight all-gathers run beside the forward GEMMs that need
            # them: those GEMMs must leave the collectives their SMs
            sms = torch.cuda.get_device_properties(self.device).multi_processor_count
            ops.set_sm_limit(self.ctx, sms - self.comm_sms)

        self.layout_ = FlatLayout(self.dims, self.world if self.sharded else 1)
        self.w_off, self.b_off = self.layout_.w_off, self.layout_.b_off
        self.n_flat = self.layout_.n_flat
        self.plan = ShardPlan(self.layout_, self.world, self.rank) if self.sharded else None
        dev = self.device

        def flat(extra=0):
            # [front slot (64 floats)] + n_flat (+ extra): every flat buffer shares
            # the gradient buffer's coordinates, so one range means the same
            # parameters in all of them (see ShardPlan)
            return torch.zeros(_LOSS_SLOTS + self.n_flat + extra, device=dev,
                               dtype=torch.float32)
        self._params_full, self._vels_full = flat(), flat()
        self.params = self._params_full[_LOSS_SLOTS:]
        self.vels = self._vels_full[_LOSS_SLOTS:]
        # grads_buf = [loss slot (64 floats)] + grads (n_flat)
        self.grads_buf = torch.zeros(self.layout_.grads_buf_len, device=dev, dtype=torch.float32)
        self.grads = self.grads_buf[_LOSS_SLOTS:]
        self.loss_slot = self.grads_buf[:1]
        if self.sharded:
            # [norm^2 partial -> global, loss partial -> global, zeros]: one small
            # all-reduce per step after the reduce-scatters
            self.scalars = torch.zeros(_ALIGN, device=dev, dtype=torch.float32)
            self.loss_slot = self.scalars[1:2]
        self.norm = torch.zeros(1, device=dev, dtype=torch.float32)
        self.w = [self._view(self.params, i, True) for i in range(self.L)]
        self.b = [self._view(self.params, i, False) for i in range(self.L)]
        self.gw = [self._view(self.grads, i, True) for i in range(self.L)]
        self.gb = [self._view(self.grads, i, False) for i in range(self.L)]
        if self.fused:
            # (+_ALIGN: every split copy keeps readable memory past its last
            # row, so MN-major tiles are fetched as whole 32-wide chunks)
            self.params_hi = flat(_ALIGN)[_LOSS_SLOTS:_LOSS_SLOTS + self.n_flat]
            self.params_lo = flat(_ALIGN)[_LOSS_SLOTS:_LOSS_SLOTS + self.n_flat]
            self.w_hi = [self._view(self.params_hi, i, True) for i in range(self.L)]
            self.w_lo = [self._view(self.params_lo, i, True) for i in range(self.L)]
        if weights is not None:
            self.load(weights, biases)
        self._bufs = {}
        self._graph = None
        # optional list; when set, each GEMM of step() appends
        # (algorithmic flops, start event, end event) -- used by the benchmark
        self.gemm_timer = None
        # optional list; when set, the split-form step appends (phase, event)
        # at its phase boundaries -- used by the benchmark
        self.phase_marks = None
        # the first layer's gradient bucket can be reduced in row chunks as
        # the chunks are computed; measured on 8 B200s this did not shorten
        # the exposed tail (the chunked GEMMs lose more than the overlap
        # gains), so one chunk is the default
        self.last_bucket_chunks = 1
        # sharded update: the first layer's weights were gathered at the end
        # of the last step
        self._gathered0 = False
        # each hidden layer's backward GEMMs (dX and dW) as one paired launch
        self.pair_backward = pair_backward is not False

    # ------------------------------------------------------------------ state
    def _wshape(self, i):
        fi, fo = self.dims[i], self.dims[i + 1]
        return (fi, fo) if self.layout == "nn" else (fo, fi)

    def _view(self, flat, i, is_w):
        if is_w:
            s = self._wshape(i)
            return flat[self.w_off[i]:self.w_off[i] + s[0] * s[1]].view(s)
        fo = self.dims[i + 1]
        return flat[self.b_off[i]:self.b_off[i] + fo]

    def load(self, weights, biases=None):
        for i in range(self.L):
            self.w[i].copy_(torch.as_tensor(np.asarray(weights[i], np.float32)).view(self._wshape(i)))
            if biases is not None:
                self.b[i].copy_(torch.as_tensor(np.asarray(biases[i], np.float32)))
        self.vels.zero_()
        if self.fused:
            ops.split_tf32(self.params, self.params_hi, self.params_lo, ctx=self.ctx)

    def weights_numpy(self):
        return ([w.detach().cpu().numpy().copy() for w in self.w],
                [b.detach().cpu().numpy().copy() for b in self.b])

    def grads_numpy(self):
        out = []
        for i in range(self.L):
            out += [self.gw[i].detach().cpu().numpy().copy(),
                    self.gb[i].detach().cpu().numpy().copy()]
        return out

    def sync_params(self, vels: bool = False):
        """Sharded update only (a collective: every rank calls it): gathers
        every rank's pieces of the parameters (and of the velocities when
        asked) so that each replica holds the full state, e.g. before reading
        or saving it.  The step itself gathers the weights it needs (the
        first layer's at the end of the previous step, the others at its
        start); between steps a rank's buffers are current only on its own
        pieces and the first layer.  No-op otherwise."""
        if not self.sharded:
            return
        bufs = [self._params_full] + ([self._vels_full] if vels else [])
        works = [self.plan.all_gather(buf, i, self.coll) for buf in bufs for i in range(self.L)]
        for wk in works:
            wk.wait()
        ops.split_tf32(self.params, self.params_hi, self.params_lo, ctx=self.ctx)

    def bucket(self, i):
        """Flat slice of grads_buf holding layer i's (dW, db); bucket 0 also
        carries the loss slot."""
        start, end = self.layout_.bucket(i)
        return self.grads_buf[start:end]

    def _buffers(self, B):
        bufs = self._bufs.get(B)
        if bufs is None:
            dev = self.device
            acts = [torch.empty((B, self.dims[i + 1]), device=dev, dtype=torch.float32)
                    for i in range(self.L)]
            gbuf = [torch.empty((B, self.dims[i + 1]), device=dev, dtype=torch.float32)
                    for i in range(self.L)]
            bufs = (acts, gbuf)
            if self.fused:
                def pair(w):  # padded past the last row (see params_hi)
                    return tuple(torch.empty(B * w + _ALIGN, device=dev,
                                             dtype=torch.float32)[:B * w].view(B, w)
                                 for _ in range(2))
                # split copies: input, hidden activations, layer gradients
                bufs = bufs + ([pair(self.dims[0])] + [pair(self.dims[i + 1])
                                                      for i in range(self.L - 1)],
                               [pair(self.dims[i + 1]) for i in range(self.L)])
                # scratch of the fused bias-gradient column sums (the CE
                # kernel's and the dX epilogues'; they run one after another
                # on the step's stream, so one buffer serves all)
                need = [ops.gemm_colsum_scratch_bytes(B, self.dims[i]) for i in range(1, self.L)]
                ce = ops.softmax_ce_colsum_scratch_bytes(B, self.dims[-1])
                self._ce_colsum = ce > 0
                nbytes = max(need + [ce, 256])
                bufs = bufs + (torch.empty(nbytes // 4 + 64, device=dev, dtype=torch.float32),)
            self._bufs[B] = bufs
        return bufs

    # ------------------------------------------------------------------ step
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        acts = self._buffers(x.shape[0])[0]
        h = x
        for i in range(self.L):
            h = ops.linear(h, self.w[i], self.b[i], relu=(i + 1 < self.L),
                           transpose_w=(self.layout == "nt"), out=acts[i],
                           ctx=self.ctx)
        return h

    def step(self, x: torch.Tensor, labels: torch.Tensor, global_batch: int | None = None,
             update: bool = True) -> torch.Tensor:
        """One training step on this rank's rows; returns the (global) loss
        as a 1-element device tensor."""
        B = x.shape[0]
        G = B * self.world if global_batch is None else int(global_batch)
        if self.fused:
            return self._step_split(x, labels, B, G, update)
        acts, gbuf = self._buffers(B)
        nt = self.layout == "nt"
        ctx = self.ctx
        timer = self.gemm_timer

        def timed(flops, fn, *a, **k):
            if timer is None:
                return fn(*a, **k)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            r = fn(*a, **k)
            e1.record()
            timer.append((flops, e0, e1))
            return r

        # forward (fused GEMM + bias + ReLU per layer)
        h = [x]
        for i in range(self.L):
            fi, fo = self.dims[i], self.dims[i + 1]
            timed(2 * B * fi * fo, ops.linear, h[i], self.w[i], self.b[i],
                  relu=(i + 1 < self.L), transpose_w=nt, out=acts[i], ctx=ctx)
            h.append(acts[i])
        # loss and dlogits in one pass; the loss lands in the first bucket
        ops.softmax_ce_labels(h[self.L], labels, denom=G, grad=gbuf[self.L - 1],
                              loss=self.loss_slot, ctx=ctx)
        works = []
        g = gbuf[self.L - 1]
        for i in reversed(range(self.L)):
            fi, fo = self.dims[i], self.dims[i + 1]
            ops.reduce_sum_leading(g, out=self.gb[i], ctx=ctx)
            if nt:   # dW[out,in] = dY^T X
                timed(2 * B * fi * fo, ops.matmul, g, h[i], fo, B, fi, ta=True, tb=False,
                      out=self.gw[i], ctx=ctx)
            else:    # dW[in,out] = X^T dY
                timed(2 * B * fi * fo, ops.matmul, h[i], g, fi, B, fo, ta=True, tb=False,
                      out=self.gw[i], ctx=ctx)
            if self.coll is not None:
                works.append(self.coll.all_reduce(self.bucket(i)))
            if i > 0:
                gprev = gbuf[i - 1]
                # dX = dY W^T: w [in,out] -> stored [N=in, K=out] (tb=1); w [out,in] -> tb=0
                timed(2 * B * fi * fo, ops.matmul, g, self.w[i], B, fo, fi, ta=False,
                      tb=not nt, out=gprev, ctx=ctx)
                ops.relu_backward(gprev, h[i], out=gprev, ctx=ctx)
                g = gprev
        for wk in works:
            wk.wait()
        if update:
            ops.sgd_momentum_autoclip(self.params, self.grads, self.vels, self.lr, self.momentum,
                                      self.weight_decay, self.max_grad_norm, norm_out=self.norm,
                                      ctx=ctx)
        return self.loss_slot

    def _step_split(self, x, labels, B, G, update):
        """The step with every GEMM operand in split form, each split copy
        written once by the kernel that produces the value: the input by one
        split pass, activations by the forward GEMM epilogue, gradients by
        the CE kernel and the dX GEMM epilogue (which also applies the ReLU
        mask of the layer below), weights by the optimizer.  Same arithmetic
        as the per-call 3xTF32 path, without its per-GEMM prepasses."""
        acts, gbuf, hsplit, gsplit, cs_scratch = self._buffers(B)
        nt = self.layout == "nt"
        ctx = self.ctx
        timer = self.gemm_timer
        d = self.dims

        def gemm(flops, **k):
            if timer is None:
                return ops.gemm_split(ctx=ctx, padded=3, **k)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            ops.gemm_split(ctx=ctx, padded=3, **k)
            e1.record()
            timer.append((flops, e0, e1))

        def gemm_pair(flops, k0, k1):
            k0, k1 = dict(k0, padded=3), dict(k1, padded=3)
            if timer is None:
                return ops.gemm_split_pair(k0, k1, ctx=ctx)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            ops.gemm_split_pair(k0, k1, ctx=ctx)
            e1.record()
            timer.append((flops, e0, e1))

        marks = self.phase_marks

        def mark(name):
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                marks.append((name, ev))

        mark("start")
        plan = self.plan
        gathers = []
        if plan is not None:
            # the new weights: every rank's pieces, layer by layer, on the
            # collective stream while the forward of the earlier layers runs
            # (the first layer's already came in at the end of the last step)
            gathers = [None if (i == 0 and self._gathered0) else self._gather_layer(i)
                       for i in range(self.L)]
            self._gathered0 = False
        xh, xl = hsplit[0]
        ops.split_tf32(x, xh, xl, ctx=ctx)
        # forward: h_{i+1} = relu(h_i W_i + b_i); split copy written by the epilogue
        for i in range(self.L):
            last = i + 1 == self.L
            if plan is not None and gathers[i] is not None:
                gathers[i].wait()
                if not self._split_on_coll_stream:
                    ops.split_tf32(self.w[i], self.w_hi[i], self.w_lo[i], ctx=ctx)
            ah, al = hsplit[i]
            ch, cl = (None, None) if last else hsplit[i + 1]
            gemm(2 * B * d[i] * d[i + 1], a_hi=ah, a_lo=al, lda=d[i], a_kmajor=True,
                 b_hi=self.w_hi[i], b_lo=self.w_lo[i], ldb=d[i] if nt else d[i + 1],
                 b_kmajor=nt, M=B, K=d[i], N=d[i + 1], c=acts[i], c_hi=ch, c_lo=cl,
                 bias=self.b[i], relu=not last)
        mark("forward")
        gh, gl = gsplit[self.L - 1]
        # the output layer's bias gradient comes out of the CE kernel, every
        # other layer's out of the dX epilogue that produces its dY
        ce_cs = self._ce_colsum
        ops.softmax_ce_labels_split(acts[self.L - 1], labels, gbuf[self.L - 1], gh, gl,
                                    self.loss_slot, G, ctx=ctx,
                                    colsum=self.gb[self.L - 1] if ce_cs else None,
                                    colsum_scratch=cs_scratch)
        mark("loss")
        works = []
        for i in reversed(range(self.L)):
            fi, fo = d[i], d[i + 1]
            g = gbuf[i]
            gh, gl = gsplit[i]
            hh, hl = hsplit[i]
            if i == self.L - 1 and not ce_cs:
                ops.reduce_sum_leading(g, out=self.gb[i], ctx=ctx)
            # dW in row chunks; with a process group, the first layer's bucket
            # (the last one backward produces, nothing left to hide it behind)
            # is all-reduced chunk by chunk as the chunks are computed
            Mrows, Ncols = (fo, fi) if nt else (fi, fo)
            nchunk = (self.last_bucket_chunks
                      if (self.coll is not None and plan is None and i == 0) else 1)
            rows_per = -(-Mrows // nchunk)
            rows_per = -(-rows_per // 128) * 128
            bstart, bend = self.layout_.bucket(i)
            dws = []  # (flops, kwargs, [lo, hi) of the gradient buffer) per row chunk
            r0 = 0
            while r0 < Mrows:
                r1 = min(Mrows, r0 + rows_per)
                if nt:   # dW[out,in] = dY^T X
                    kw = dict(a_hi=gh.view(-1)[r0:], a_lo=gl.view(-1)[r0:], lda=fo,
                              a_kmajor=False, b_hi=hh, b_lo=hl, ldb=fi, b_kmajor=False,
                              M=r1 - r0, K=B, N=fi, c=self.gw[i].view(-1)[r0 * Ncols:], ldc=Ncols)
                else:    # dW[in,out] = X^T dY
                    kw = dict(a_hi=hh.view(-1)[r0:], a_lo=hl.view(-1)[r0:], lda=fi,
                              a_kmajor=False, b_hi=gh, b_lo=gl, ldb=fo, b_kmajor=False,
                              M=r1 - r0, K=B, N=fo, c=self.gw[i].view(-1)[r0 * Ncols:], ldc=Ncols)
                lo = bstart if r0 == 0 else _LOSS_SLOTS + self.w_off[i] + r0 * Ncols
                hi = bend if r1 == Mrows else _LOSS_SLOTS + self.w_off[i] + r1 * Ncols
                dws.append((2 * B * (r1 - r0) * Ncols, kw, lo, hi))
                r0 = r1
            dx = None
            if i > 0:
                # dX = (dY W^T) masked by relu'(h_i); split copy for the next GEMMs
                ph, pl = gsplit[i - 1]
                dx = (2 * B * fi * fo,
                      dict(a_hi=gh, a_lo=gl, lda=fo, a_kmajor=True, b_hi=self.w_hi[i],
                           b_lo=self.w_lo[i], ldb=fi if nt else fo, b_kmajor=not nt, M=B, K=fo,
                           N=fi, c=gbuf[i - 1], c_hi=ph, c_lo=pl, mask=acts[i - 1], ldm=fi,
                           colsum=self.gb[i - 1], colsum_scratch=cs_scratch))
            if dx is not None and len(dws) == 1 and self.pair_backward:
                # dX and dW read the same dY and not each other: one launch
                gemm_pair(dx[0] + dws[0][0], dx[1], dws[0][1])
                dx = None
            else:
                for fl, kw, lo, hi in dws:
                    gemm(fl, **kw)
                    if self.coll is not None and nchunk > 1:
                        works.append(self.coll.all_reduce(self.grads_buf[lo:hi]))
            # the first layer's bucket comes last: nothing is left to overlap it
            if plan is not None:
                works.append(plan.reduce_scatter(self.grads_buf, i, self.coll, overlap=i > 0))
            elif self.coll is not None and nchunk == 1:
                works.append(self.coll.all_reduce(self.bucket(i), overlap=i > 0))
            if dx is not None:
                gemm(dx[0], **dx[1])
        mark("backward")
        for wk in works:
            wk.wait()
        mark("allreduce_wait")
        if plan is not None:
            self._sharded_update(update)
        elif update:
            ops.sgd_momentum_autoclip_split(self.params, self.grads, self.vels, self.params_hi,
                                            self.params_lo, self.lr, self.momentum,
                                            self.weight_decay, self.max_grad_norm,
                                            norm_out=self.norm, ctx=ctx)
        mark("update")
        return self.loss_slot

    @property
    def _split_on_coll_stream(self):
        return getattr(self.coll, "stream", None) is not None

    def _gather_layer(self, i):
        """Sharded update: all-gather layer i's new weights (every rank's
        pieces) and, where the collectives run on a stream of their own,
        re-split them to hi/lo right behind the gather on that stream -- the
        split then runs on the SMs the GEMMs leave free, beside the forward
        of the earlier layers, instead of in front of layer i's GEMM."""
        # the first layer's gather runs where nothing overlaps it
        work = self.plan.all_gather(self._params_full, i, self.coll, overlap=i > 0)
        if not self._split_on_coll_stream:
            return work
        from .collectives import _EventWork
        with torch.cuda.stream(self.coll.stream):
            ops.split_tf32(self.w[i], self.w_hi[i], self.w_lo[i], ctx=self.ctx)
            ev = torch.cuda.Event()
            ev.record(self.coll.stream)
        return _EventWork(ev)

    def _sharded_update(self, update):
        """Global norm from every rank's gradient pieces (one small
        all-reduce that also sums the loss), then the update of this rank's
        pieces.  The first layer's new weights are all-gathered (and
        re-split) right after its piece is updated, beside the update of the
        other pieces: the next step's first GEMM needs them before anything
        else could hide the gather.  The other layers' weights are gathered
        at the next step's start, beside its forward."""
        ranges = self.plan.update_ranges()
        sc = self.scalars
        if ranges:
            for k, (a, b) in enumerate(ranges):
                ops.sum_squares(self.grads_buf[a:b], sc[0:1], accumulate=k > 0, ctx=self.ctx)
        else:
            ops.sum_squares(self.grads_buf[:0], sc[0:1], ctx=self.ctx)
        self.coll.all_reduce(sc, overlap=False).wait()
        if not update:
            return
        g0 = None
        for i, (a, b) in enumerate(self.plan.pieces):
            a = max(a, _LOSS_SLOTS)
            if b > a:
                ops.sgd_momentum_clip(self._params_full[a:b], self.grads_buf[a:b],
                                      self._vels_full[a:b], self.lr, self.momentum,
                                      self.weight_decay, self.max_grad_norm, sc[0:1],
                                      ctx=self.ctx)
            if i == 0:
                g0 = self._gather_layer(0)
        g0.wait()
        if not self._split_on_coll_stream:
            ops.split_tf32(self.w[0], self.w_hi[0], self.w_lo[0], ctx=self.ctx)
        self._gathered0 = True

    # ------------------------------------------------------------ CUDA graph
    def capture(self, x: torch.Tensor, labels: torch.Tensor, global_batch: int | None = None):
        """Captures one full step (including the all-reduces) into a CUDA
        graph reading from the given input buffers.  Run a step eagerly first
        so every workspace is sized."""
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step(x, labels, global_batch)
        self._graph = g
        return g

    def replay(self):
        self._graph.replay()
        return self.loss_slot

    def release_graph(self):
        self._graph = None

    def close(self):
        """Releases the captured step and, when this model made its own NCCL
        communicator, destroys it (every rank calls close; graphs holding
        its collectives go first)."""
        self._graph = None
        if self.coll is not None and self._owns_coll:
            self.coll.destroy()
        self.coll = None
        if self.ctx:
            ops.destroy_context(self.ctx)
            self.ctx = None


class HostBatchPipeline:
    """Trains an MLP from batches in pinned host memory: while one step runs,
    the next batch is copied to the device on a separate stream, into the
    other of two device buffers (with CUDA graphs, one captured step per
    buffer); each step's loss is read back to the host.  This replaces the
    reference's synchronous upload (`GpuTensor::from_host`,
    moonxi-net-gpu/tensor/gpu_tensor.mbt:192-211, driven by the data loader
    moonxi-net/datasets/mnist/mnist.mbt:167-183) with copies that overlap the
    previous step.

    Run one eager step of the model first (it sizes every workspace) before
    building the pipeline with `use_graph=True`.  A batch's host memory must
    stay unchanged until `run` returns.
    """

    def __init__(self, model: MLP, rows: int, global_batch: int | None = None,
                 use_graph: bool = True):
        dev = model.device
        self.model = model
        self.global_batch = global_batch
        self.x = [torch.empty((rows, model.dims[0]), device=dev, dtype=torch.float32)
                  for _ in range(2)]
        self.y = [torch.empty(rows, device=dev, dtype=torch.float32) for _ in range(2)]
        self.copy_stream = torch.cuda.Stream(device=dev)
        self.ready = [torch.cuda.Event(), torch.cuda.Event()]   # batch uploaded
        self.done = [torch.cuda.Event(), torch.cuda.Event()]    # step using the buffer ended
        self.loss_ready = [torch.cuda.Event(), torch.cuda.Event()]
        self.loss_host = torch.zeros(2, dtype=torch.float32).pin_memory()
        self.graphs = None
        if use_graph:
            self.graphs = [model.capture(self.x[i], self.y[i], global_batch) for i in range(2)]

    def _upload(self, slot, x, y, after=None):
        with torch.cuda.stream(self.copy_stream):
            if after is not None:  # the buffer's previous step must be done with it
                self.copy_stream.wait_event(after)
            self.x[slot].copy_(x, non_blocking=True)
            self.y[slot].copy_(y, non_blocking=True)
            self.ready[slot].record(self.copy_stream)

    def run(self, batches) -> list[float]:
        """One training step per (x, y) host batch; returns the losses.

        Nothing on the host waits for a step before the next one is queued:
        the upload into a buffer waits on the GPU for the step that last read
        it, each step's loss is copied to pinned host memory as the step
        ends, and the host reads step i's loss while step i+1 runs."""
        losses = []
        it = iter(batches)
        cur_batch = next(it, None)
        if cur_batch is None:
            return losses
        compute = torch.cuda.current_stream()
        self._upload(0, *cur_batch)
        i, pending = 0, None
        while cur_batch is not None:
            cur = i % 2
            nxt_batch = next(it, None)
            if nxt_batch is not None:
                self._upload(1 - cur, *nxt_batch, after=self.done[1 - cur] if i >= 1 else None)
            compute.wait_event(self.ready[cur])
            if self.graphs is not None:
                self.graphs[cur].replay()
            else:
                self.model.step(self.x[cur], self.y[cur], self.global_batch)
            self.done[cur].record(compute)
            self.loss_host[cur:cur + 1].copy_(self.model.loss_slot, non_blocking=True)
            self.loss_ready[cur].record(compute)
            if pending is not None:  # step i-1's loss, read while step i runs
                self.loss_ready[pending].synchronize()
                losses.append(float(self.loss_host[pending]))
            pending = cur
            cur_batch = nxt_batch
            i += 1
        self.loss_ready[pending].synchronize()
        losses.append(float(self.loss_host[pending]))
        return losses

    def release(self):
        """Drops the captured graphs (before the process group goes, when
        they hold collectives)."""
        self.graphs = None
        self.model.release_graph()
