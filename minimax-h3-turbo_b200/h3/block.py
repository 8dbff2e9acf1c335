"""One single-stream H3 DiT block driven through the W4A8 kernels, optionally token-sharded across GPUs.

Semantics of the reference block (h3turbo/h3/model.py:_block :234-242, _attention :196-228, _mlp :186-194 with
_rms / _scale_shift_ / _gate_ :64-115 and q/k norm + split-half RoPE, layout.py:norm_rope_ :329-356 in its "torch" form
:309-326): with AdaLN modulation rows per token segment (precomputed here, as the benchmark configuration states),

    h = rms(x, norm1) * (1 + sc_a) + sh_a                (bf16)
    q, k, v = qlinear(h, qkv);  q, k <- rope(rms_h(q)), rope(rms_h(k));  o = sdpa(q, k, v)
    x = x + g_a * qlinear(o, out)
    h = rms(x, norm2) * (1 + sc_m) + sh_m
    x = x + g_m * qlinear(qlinear(h, fc1), fc2, input_act="swiglu")

Every linear is the W4A8 qlinear (kernels KA + KB, with the RMSNorm + modulation fused into the quantiser of qkv and
fc1); q/k norm + RoPE, the modulation and the gated residuals are this library's fused kernels; attention is torch's
fused SDPA library kernel (cuDNN on B200, bf16).  The operators live in `KernelOps`, which refuses CPU and fp32
tensors: there is no CPU path.  (The token-sharding tests run the same block on CPU ranks by passing their own
operator set, written with the reference's torch formulas, as `ops=`.)

Token sharding (rank r of P owns a contiguous slice of rows): every op above is token-wise except attention, which needs
all keys and values.  kv_exchange "gather" (the default) all-gathers K and V and makes one attention call over all
keys: every query sees exactly what it would see on one GPU, so the sharded block is bit-identical to the unsharded one.
"overlap" sends this rank's keys and values to every other rank and receives theirs (NCCL point-to-point, one batched
group) while the local queries attend to the local keys; one attention call over the received keys follows, and the two
partial results are merged by their log-sum-exps (h3b_attn_merge) -- the exchange hides behind 1/P of the attention,
at the price of two attention calls and results that differ from one call in the last bits.  "ring" passes the shards
round the ranks.  `gather_rows` assembles the final hidden states at the sequence boundary.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from . import qlinear as ql
from .rope import norm_rope_
from .types import BlockWeights

Segment = Tuple[int, int, int]  # (first row, end row, modulation row)


def _aligned_rows(t: torch.Tensor) -> torch.Tensor:
    """t itself when it is a row-major 2-D view the kernels can read (16-byte aligned, row stride a multiple of 8)."""
    ok = t.dim() == 2 and t.stride(1) == 1 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0
    return t if ok else t.contiguous()


def _segment_args(segments: Sequence[Segment], m: int, n_rows: int, device):
    """(host int32 table or None, its length, device per-token row map or None) for the modulation kernels: up to 16
    segments with int rows go by value; more, or per-token row tensors (the reference's _pieces), use a row map."""
    import ctypes

    segs = [(a, b, r) for a, b, r in segments if b > a]
    if len(segs) <= 16 and all(isinstance(r, int) for _, _, r in segs):
        for a, b, r in segs:
            if not 0 <= r < n_rows or a < 0 or b > m:
                raise ValueError(f"segment {(a, b, r)} is out of range for {m} tokens and {n_rows} modulation rows")
        return (ctypes.c_int32 * max(1, 3 * len(segs)))(*[v for seg in segs for v in seg]), len(segs), None
    rows = torch.full((m,), -1, dtype=torch.int32, device=device)
    for a, b, r in segs:
        rows[a:b] = r.to(device=device, dtype=torch.int32) if isinstance(r, torch.Tensor) else int(r)
    return None, 0, rows


def _kernel_rows(x: torch.Tensor) -> bool:
    return x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and x.dim() == 2 and x.shape[1] % 8 == 0


def _require_kernel_rows(x: torch.Tensor, what: str) -> None:
    if not _kernel_rows(x):
        raise RuntimeError(f"{what}: the b200 kernels take bf16/fp16 CUDA rows with a width that is a multiple of 8, got "
                           f"{tuple(x.shape)} {x.dtype} on {x.device} (there is no CPU or fp32 path)")


def rms_modulate(x: torch.Tensor, weight: torch.Tensor, eps: float, shift: torch.Tensor, scale: torch.Tensor,
                 segments: Sequence[Segment]) -> torch.Tensor:
    """h = _scale_shift_(_rms(x, weight, eps), shift, scale, segments) as one pass over x (model.py:64-66, 106-109) on
    the fused kernel, for bf16/fp16 CUDA rows (segment rows: ints, or int tensors of per-token rows as the reference's
    _pieces takes).  Other tensors raise RuntimeError."""
    _require_kernel_rows(x, "rms_modulate")
    from .. import _lib

    m, hid = x.shape
    x = _aligned_rows(x)
    shift, scale = _aligned_rows(shift), _aligned_rows(scale)
    if scale.dtype != shift.dtype:
        scale = scale.to(shift.dtype)
    if shift.stride(0) != scale.stride(0) or shift.shape != scale.shape or shift.shape[1] != hid:
        shift, scale = shift.contiguous(), scale.contiguous()
    w = weight.contiguous()
    n_rows = shift.shape[0]
    table, n_seg, token_rows = _segment_args(segments, m, n_rows, x.device)
    h = torch.empty(m, hid, dtype=x.dtype, device=x.device)
    L = _lib.lib()
    _lib.check(L.h3b_rms_modulate(x.data_ptr(), _lib.act_code(x.dtype), x.stride(0), m, hid, w.data_ptr(),
                                  _lib.act_code(w.dtype), float(eps), shift.data_ptr(), scale.data_ptr(), shift.stride(0),
                                  n_rows, _lib.act_code(shift.dtype), table, n_seg, _lib.ptr(token_rows), h.data_ptr(), hid,
                                  _lib.stream_ptr(x.device)), "rms_modulate")
    return h


class Prenorm:
    """x with its block's RMSNorm + modulation still pending: h = scale_shift_(rms(x, weight, eps), shift, scale,
    segments) (model.py:64-66, 106-109, 239-241).  The W4A8 linear that reads h takes it through the fused
    norm + rotate + quantise kernel (prenorm_linear), so h never goes to memory; materialize() computes h."""

    def __init__(self, x: torch.Tensor, weight: torch.Tensor, eps: float, shift: torch.Tensor, scale: torch.Tensor,
                 segments: Sequence[Segment]):
        self.x, self.weight, self.eps, self.shift, self.scale, self.segments = x, weight, eps, shift, scale, segments

    @property
    def shape(self):
        return self.x.shape

    @property
    def dtype(self):
        return self.x.dtype

    @property
    def device(self):
        return self.x.device

    def materialize(self) -> torch.Tensor:
        return rms_modulate(self.x, self.weight, self.eps, self.shift, self.scale, self.segments)


def prenorm_codes(pre: Prenorm, convrot: int = 256, quant_mode: str = "ck") -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
    """(int8 codes [M, K], fp32 scales [M, 1]) of h = pre.materialize() from the fused kernel (h3b_rotq_rms_modulate),
    bit-identical to quantising the materialised h; None where that kernel does not apply (not bf16 CUDA rows, K not a
    multiple of 256 or above 6144, ConvRot other than 256)."""
    x = pre.x
    if not (x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.shape[1] % 256 == 0 and x.shape[1] <= 6144
            and convrot == 256):
        return None
    from .. import _lib

    m, k = x.shape
    x = _aligned_rows(x)
    bf = torch.bfloat16
    shift = pre.shift.to(bf)  # dt(shift[row]) and dt(1 + dt(scale[row])): what _scale_shift_ adds and multiplies by
    scale1 = (1.0 + pre.scale.to(bf)).to(bf)
    shift, scale1 = shift.contiguous(), scale1.contiguous()
    if shift.shape != scale1.shape or shift.shape[-1] != k:
        raise ValueError(f"shift / scale must be [rows, {k}], got {tuple(pre.shift.shape)} / {tuple(pre.scale.shape)}")
    w = pre.weight.to(bf).contiguous()
    n_rows = shift.shape[0]
    table, n_seg, token_rows = _segment_args(pre.segments, m, n_rows, x.device)
    q = torch.empty(m, k, dtype=torch.int8, device=x.device)
    xs = torch.empty(m, 1, dtype=torch.float32, device=x.device)
    L = _lib.lib()
    _lib.check(L.h3b_rotq_rms_modulate(x.data_ptr(), m, k, x.stride(0), w.data_ptr(), float(pre.eps), shift.data_ptr(),
                                       scale1.data_ptr(), shift.stride(0), n_rows, table, n_seg, _lib.ptr(token_rows),
                                       convrot, _lib.QMODE[quant_mode], q.data_ptr(), k, xs.data_ptr(),
                                       _lib.stream_ptr(x.device)), "rotq_rms_modulate")
    return q, xs


def prenorm_linear(pre: Prenorm, w, precision: str = "a8", quant_mode: str = "ck") -> torch.Tensor:
    """linear(pre.materialize(), w) with the norm fused into the quantiser when it applies (W4A8 weight, a8)."""
    if isinstance(w, ql.W4A8Weight) and precision == "a8" and pre.x.shape[0] > 0:
        codes = prenorm_codes(pre, w.convrot, quant_mode)
        if codes is not None:
            if w.q.shape[1] * 2 != pre.x.shape[1]:
                raise ValueError(f"input features {pre.x.shape[1]} do not match the weight's K={w.q.shape[1] * 2}")
            return ql._gemm_codes(codes[0], codes[1], w, None, out_dtype=pre.x.dtype, quant_mode=quant_mode)
    return ql.linear(pre.materialize(), w, precision=precision, quant_mode=quant_mode)


def gate_(x: torch.Tensor, gate: torch.Tensor, other: torch.Tensor, segments: Sequence[Segment]) -> torch.Tensor:
    """x[a:b] += other[a:b] * gate[row] per segment, in place (model.py:111-115), on the fused kernel (bit-identical to
    torch's addcmul_) for bf16/fp16 CUDA rows; x must be a row-major view with 16-byte aligned rows."""
    _require_kernel_rows(x, "gate_")
    if other.shape != x.shape or other.dtype != x.dtype or x.stride(1) != 1 or x.stride(0) % 8 or x.data_ptr() % 16:
        raise ValueError("gate_: other must match x, and x must be row-major with 16-byte aligned rows")
    from .. import _lib

    m, hid = x.shape
    other, g = _aligned_rows(other), _aligned_rows(gate)
    table, n_seg, token_rows = _segment_args(segments, m, g.shape[0], x.device)
    _lib.check(_lib.lib().h3b_gate_residual(x.data_ptr(), _lib.act_code(x.dtype), x.stride(0), other.data_ptr(),
                                            other.stride(0), m, hid, g.data_ptr(), g.stride(0), g.shape[0],
                                            _lib.act_code(g.dtype), table, n_seg, _lib.ptr(token_rows),
                                            _lib.stream_ptr(x.device)), "gate_residual")
    return x


@dataclass
class Modulation:
    """AdaLN outputs of one block: six [rows, hidden] tensors (model.py:230-232)."""

    shift_a: torch.Tensor
    scale_a: torch.Tensor
    gate_a: torch.Tensor
    shift_m: torch.Tensor
    scale_m: torch.Tensor
    gate_m: torch.Tensor


@dataclass
class ShardSpec:
    """Token sharding: this rank owns rows [start, stop) of `total`; `group` is the process group (None = one GPU)."""

    start: int
    stop: int
    total: int
    group: Optional[object] = None
    world: int = 1
    rank: int = 0


def shard_rows(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous balanced split: the first total % world ranks get one extra row."""
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_rows(x: torch.Tensor, spec: ShardSpec) -> torch.Tensor:
    """All-gather of row shards -> [total, ...] on every rank (NCCL all_gather of equal-size, padded buffers)."""
    return gather_rows_async(x, spec)()


def gather_rows_async(x: torch.Tensor, spec: ShardSpec):
    """Starts gather_rows(x, spec) and returns a function that waits for it (on the caller's stream, for NCCL) and
    returns the gathered rows: the collective runs while the caller queues other work."""
    if spec.group is None or spec.world == 1:
        return lambda: x
    import torch.distributed as dist

    sizes = [b - a for a, b in (shard_rows(spec.total, spec.world, r) for r in range(spec.world))]
    cap = max(sizes)
    if x.shape[0] == cap and x.is_contiguous():
        buf = x
    else:
        buf = torch.empty(cap, *x.shape[1:], dtype=x.dtype, device=x.device)
        buf[: x.shape[0]] = x
    out = torch.empty(spec.world * cap, *x.shape[1:], dtype=x.dtype, device=x.device)
    if dist.get_backend(spec.group) == "nccl":
        work = dist.all_gather_into_tensor(out, buf, group=spec.group, async_op=True)
    else:  # gloo (CPU ranks): list form
        work = dist.all_gather(list(out.chunk(spec.world)), buf, group=spec.group, async_op=True)

    def finish() -> torch.Tensor:
        work.wait()
        if all(n == cap for n in sizes):
            return out
        return torch.cat([out[r * cap: r * cap + sizes[r]] for r in range(spec.world)])

    return finish


def attention_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Softmax attention of q [1, H, Sq, D] over k, v [1, H, Sk, D] -> (o [1, H, Sq, D] in q.dtype, lse [1, H, Sq] fp32,
    the natural-log sum of exp of the scaled scores), through torch's cuDNN fused attention.  CUDA tensors only."""
    if not q.is_cuda:
        raise RuntimeError("attention_lse: CUDA tensors only (there is no CPU path)")
    r = torch.ops.aten._scaled_dot_product_cudnn_attention(q, k, v, None, True)
    return r[0], r[1].reshape(q.shape[:-1]).to(torch.float32)


class AttnMerger:
    """Folds softmax attention over disjoint key sets into one result with the merge kernel (h3b_attn_merge): add()
    the (o [1, H, S, D] bf16, lse [1, H, S] fp32) of each key set in turn; the call with last=True returns the merged
    [S, H * D] bf16 rows (the layout the output projection reads).  A key set without keys has lse -inf (weight 0)."""

    def __init__(self, heads: int, queries: int, head_dim: int, device):
        self.h, self.s, self.d = heads, queries, head_dim
        self.acc = torch.empty(heads, queries, head_dim, dtype=torch.float32, device=device)
        self.acc_lse = torch.empty(heads, queries, dtype=torch.float32, device=device)
        self.n = 0

    def add(self, o: torch.Tensor, lse: torch.Tensor, last: bool = False) -> Optional[torch.Tensor]:
        from .. import _lib

        if o.dtype != torch.bfloat16 or not o.is_cuda:
            raise RuntimeError("AttnMerger: bf16 CUDA attention outputs only")
        if o.stride(3) != 1:
            o = o.contiguous()
        lse = lse.reshape(self.h, self.s).contiguous()
        out = torch.empty(self.s, self.h * self.d, dtype=o.dtype, device=o.device) if last else None
        _lib.check(_lib.lib().h3b_attn_merge(self.acc.data_ptr(), self.acc_lse.data_ptr(), o.data_ptr(), o.stride(1),
                                             o.stride(2), _lib.BF16, lse.data_ptr(), self.h, self.s, self.d,
                                             int(self.n == 0), _lib.ptr(out), self.h * self.d,
                                             _lib.stream_ptr(o.device)), "attn_merge")
        self.n += 1
        return out


class KernelOps:
    """The block's operators on this library's kernels and torch's fused attention: bf16/fp16 CUDA tensors only."""

    @staticmethod
    def rms_modulate(x, weight, eps, shift, scale, segments):
        return rms_modulate(x, weight, eps, shift, scale, segments)

    @staticmethod
    def gate_(x, gate, other, segments):
        return gate_(x, gate, other, segments)

    @staticmethod
    def norm_rope_(q, k, wq, wk, eps, cos, sin):
        norm_rope_(q, k, wq, wk, eps, cos, sin, impl="b200")

    @staticmethod
    def attention(q, k, v):
        if not q.is_cuda:
            raise RuntimeError("attention: CUDA tensors only (there is no CPU path)")
        return F.scaled_dot_product_attention(q, k, v)

    @staticmethod
    def attention_lse(q, k, v):
        return attention_lse(q, k, v)

    @staticmethod
    def merger(heads, queries, head_dim, device):
        return AttnMerger(heads, queries, head_dim, device)


KERNEL_OPS = KernelOps()


def _heads_first(t: torch.Tensor) -> torch.Tensor:
    """[S, H, D] (any row stride) -> the [1, H, S, D] view attention takes."""
    return t.transpose(0, 1).unsqueeze(0)


def _empty_part(h: int, s: int, d: int, like: torch.Tensor):
    """(o, lse) of attention over an empty key set: zeros and -inf."""
    return (torch.zeros(1, h, s, d, dtype=like.dtype, device=like.device),
            torch.full((1, h, s), float("-inf"), dtype=torch.float32, device=like.device))


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, spec: ShardSpec, ops=KERNEL_OPS) -> torch.Tensor:
    """Attention of this rank's queries over every rank's keys and values, with the key/value shards passed round a
    ring of the ranks (P - 1 point-to-point steps) while the attention over the shard already here runs: the transfer
    of step s + 1 overlaps the attention of step s.  q, k, v: [S_local, H, D]; returns [S_local, H * D] in q.dtype."""
    import torch.distributed as dist

    p_, r_ = spec.world, spec.rank
    sizes = [b - a for a, b in (shard_rows(spec.total, p_, i) for i in range(p_))]
    cap = max(sizes)
    s, h, d = k.shape
    bufs = [torch.zeros(2, cap, h, d, dtype=k.dtype, device=k.device) for _ in range(2)]
    bufs[0][0, :s] = k
    bufs[0][1, :s] = v
    qh = _heads_first(q)
    merger = ops.merger(h, s, d, q.device)
    nxt, prv = (r_ + 1) % p_, (r_ - 1) % p_
    out = None
    for step in range(p_):
        cur = bufs[step % 2]
        reqs = []
        if step < p_ - 1:
            reqs = dist.batch_isend_irecv([dist.P2POp(dist.isend, cur, nxt, group=spec.group),
                                           dist.P2POp(dist.irecv, bufs[(step + 1) % 2], prv, group=spec.group)])
        n = sizes[(r_ - step) % p_]  # the shard in `cur` came from rank r - step
        if n == 0 or s == 0:  # an empty shard (fewer tokens than ranks) has no keys
            o, lse = _empty_part(h, s, d, q)
        else:
            o, lse = ops.attention_lse(qh, _heads_first(cur[0, :n]), _heads_first(cur[1, :n]))
        out = merger.add(o, lse, last=step == p_ - 1)
        for rq in reqs:
            rq.wait()
    return out


def overlap_attention(q: torch.Tensor, kv: torch.Tensor, spec: ShardSpec, ops=KERNEL_OPS,
                      probe: Optional[Callable[[str], None]] = None) -> torch.Tensor:
    """Attention of this rank's queries over every rank's keys and values, the exchange hidden behind the local part.

    kv: [S_local, 2 * H * D] rows of this rank's keys then values (the q/k-normalised K | V half of the qkv output).
    This rank's rows go to every other rank and theirs arrive in one buffer, ordered r + 1, r + 2, ..., r - 1 and
    packed without gaps (one batched group of NCCL point-to-point transfers); meanwhile the local queries attend to the
    local keys.  One attention call over all received keys follows, and the merge kernel folds the two partial results
    by their log-sum-exps.  q: [S_local, H, D]; returns [S_local, H * D] in q.dtype."""
    import torch.distributed as dist

    p_, r_ = spec.world, spec.rank
    s, h, d = q.shape
    inner = h * d
    sizes = [b - a for a, b in (shard_rows(spec.total, p_, i) for i in range(p_))]
    peers = [(r_ + i) % p_ for i in range(1, p_)]
    kv = kv.contiguous()
    remote = torch.empty(spec.total - s, 2 * inner, dtype=kv.dtype, device=kv.device)
    p2p, off = [], 0
    for j in peers:
        if s > 0:
            p2p.append(dist.P2POp(dist.isend, kv, j, group=spec.group))
        if sizes[j] > 0:
            p2p.append(dist.P2POp(dist.irecv, remote[off:off + sizes[j]], j, group=spec.group))
        off += sizes[j]
    reqs = dist.batch_isend_irecv(p2p) if p2p else []
    qh = _heads_first(q)
    merger = ops.merger(h, s, d, q.device)
    if s > 0:
        o, lse = ops.attention_lse(qh, _heads_first(kv[:, :inner].view(s, h, d)), _heads_first(kv[:, inner:].view(s, h, d)))
    else:
        o, lse = _empty_part(h, s, d, q)
    merger.add(o, lse)
    if probe:
        probe("local_done")
    for rq in reqs:
        rq.wait()
    if probe:
        probe("kv_ready")
    n = remote.shape[0]
    if n > 0 and s > 0:
        o, lse = ops.attention_lse(qh, _heads_first(remote[:, :inner].view(n, h, d)),
                                   _heads_first(remote[:, inner:].view(n, h, d)))
    else:
        o, lse = _empty_part(h, s, d, q)
    return merger.add(o, lse, last=True)


KV_EXCHANGES = ("gather", "overlap", "ring")


class DiTBlock:
    """Runs H3 DiT blocks on the W4A8 kernels.  heads / head_dim / eps as in H3Config.

    kv_exchange (token-sharded runs): "gather" (default: one all-gather of K and V, optionally in `kv_groups` head
    groups, then one attention call; bit-identical to one GPU), "overlap" (keys and values exchanged point-to-point
    while the local queries attend to the local keys, then one call over the received keys and a log-sum-exp merge) or
    "ring" (shards passed round the ranks, one attention call and merge per shard).  `ops`: the operator set (KernelOps; tests of the
    sharding plumbing on CPU ranks pass the reference's torch formulas).  `probe(tag)`, when given, is called on the
    host at the phase boundaries of the attention ("qk_ready", "local_done", "kv_ready", "attn_done") so a caller can
    record CUDA events there."""

    def __init__(self, heads: int, head_dim: int, norm_eps: float = 1e-5, qk_norm_eps: float = 1e-5,
                 precision: str = "a8", attn_chunk: Optional[int] = None, linear=None, kv_exchange: str = "gather",
                 fuse_norm: Optional[bool] = None, kv_groups: int = 1, ops=None,
                 probe: Optional[Callable[[str], None]] = None):
        if kv_exchange not in KV_EXCHANGES:
            raise ValueError(f"kv_exchange must be one of {KV_EXCHANGES}, got {kv_exchange!r}")
        if kv_groups < 1:
            raise ValueError(f"kv_groups must be >= 1, got {kv_groups}")
        self.kv_exchange = kv_exchange
        self.kv_groups = kv_groups
        self.heads, self.head_dim = heads, head_dim
        self.norm_eps, self.qk_norm_eps, self.precision = norm_eps, qk_norm_eps, precision
        self.attn_chunk = attn_chunk
        self.ops = ops or KERNEL_OPS
        self.probe = probe
        # the linear op: the W4A8 qlinear (default); tests of the token-sharding plumbing on CPU ranks pass a dense one
        self._linear = linear or (lambda x, w, input_act=None: ql.linear(x, w, precision=self.precision, input_act=input_act))
        self._linear_is_default = linear is None
        # RMSNorm + modulation fused into the quantiser of the qkv and fc1 linears: on for the default linear; a custom
        # linear opts in with fuse_norm=True and then receives a Prenorm for those two
        self._fuse_norm = linear is None if fuse_norm is None else fuse_norm

    def _mark(self, tag: str) -> None:
        if self.probe:
            self.probe(tag)

    def _in_linear(self, h, w) -> torch.Tensor:
        """The linear that reads the normalised stream (qkv, fc1): h is a tensor or a Prenorm."""
        if isinstance(h, Prenorm) and self._linear_is_default:
            return prenorm_linear(h, w, self.precision)
        return self._linear(h, w)

    def attention(self, h: torch.Tensor, w: BlockWeights, cos: torch.Tensor, sin: torch.Tensor,
                  spec: Optional[ShardSpec] = None) -> torch.Tensor:
        s, heads, hd = h.shape[0], self.heads, self.head_dim
        inner = heads * hd
        qkv = self._in_linear(h, w.qkv)
        q, k, v = (t.view(s, heads, hd) for t in qkv.split(inner, dim=-1))
        self.ops.norm_rope_(q, k, w.q_norm, w.k_norm, self.qk_norm_eps, cos, sin)
        self._mark("qk_ready")
        sharded = spec is not None and spec.world > 1
        if sharded and self.kv_exchange == "overlap":
            o = overlap_attention(q, qkv[:, inner:], spec, self.ops, self.probe)
            self._mark("attn_done")
            return self._linear(o, w.out)
        if sharded and self.kv_exchange == "ring":
            o = ring_attention(q, k, v, spec, self.ops)
            self._mark("attn_done")
            return self._linear(o, w.out)
        if sharded:  # "gather": every query needs every key and value
            groups = self.kv_groups if heads % self.kv_groups == 0 and not (self.attn_chunk and self.attn_chunk < s) else 1
            if groups > 1:
                o = self._grouped_gather_attention(q, k, v, spec, groups)
                self._mark("attn_done")
                return self._linear(o, w.out)
            k = gather_rows(k.reshape(s, inner).contiguous(), spec).view(-1, heads, hd)
            v = gather_rows(v.reshape(s, inner).contiguous(), spec).view(-1, heads, hd)
            self._mark("kv_ready")
        qh, kh, vh = _heads_first(q), _heads_first(k), _heads_first(v)
        step = self.attn_chunk or s
        if step >= s:
            o = self.ops.attention(qh, kh, vh).transpose(1, 2).reshape(s, inner)
        else:  # query rows are independent (chunks may pick another attention kernel: not bit-identical)
            o = torch.empty(s, inner, dtype=h.dtype, device=h.device)
            for a in range(0, s, step):
                o[a:a + step] = self.ops.attention(qh[:, :, a:a + step], kh, vh)[0].transpose(0, 1).reshape(-1, inner)
        self._mark("attn_done")
        return self._linear(o, w.out)

    def _grouped_gather_attention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, spec: ShardSpec,
                                  groups: int) -> torch.Tensor:
        """Attention of the local queries over all ranks' keys and values, gathered in `groups` head groups: every
        group's K and V all-gathers are started first, then each group's attention waits only for its own.  At config
        5 on 2 B200s this measured slower than one all-gather (157.2 vs 152.5 ms per forward: four smaller attention
        calls cost more than the hidden transfer)."""
        s, heads, hd = q.shape
        hg = heads // groups
        pending = []
        for g in range(groups):
            h0 = g * hg
            kl = k[:, h0:h0 + hg].reshape(s, hg * hd).contiguous()
            vl = v[:, h0:h0 + hg].reshape(s, hg * hd).contiguous()
            pending.append((gather_rows_async(kl, spec), gather_rows_async(vl, spec)))
        o = torch.empty(s, heads * hd, dtype=q.dtype, device=q.device)
        for g, (kf, vf) in enumerate(pending):
            h0 = g * hg
            kg, vg = kf().view(-1, hg, hd), vf().view(-1, hg, hd)
            o[:, h0 * hd:(h0 + hg) * hd] = self.ops.attention(_heads_first(q[:, h0:h0 + hg]), _heads_first(kg),
                                                              _heads_first(vg))[0].transpose(0, 1).reshape(s, hg * hd)
        return o

    def mlp(self, h: torch.Tensor, w: BlockWeights) -> torch.Tensor:
        return self._linear(self._in_linear(h, w.fc1), w.fc2, input_act="swiglu")

    def __call__(self, x: torch.Tensor, w: BlockWeights, mod: Modulation, segments: Sequence[Segment], cos: torch.Tensor,
                 sin: torch.Tensor, spec: Optional[ShardSpec] = None) -> torch.Tensor:
        """x: [S_local, hidden] residual stream (updated in place and returned); cos/sin: [S_local, half] for these rows."""
        norm = Prenorm if self._fuse_norm else self.ops.rms_modulate
        h = norm(x, w.norm1, self.norm_eps, mod.shift_a, mod.scale_a, segments)
        self.ops.gate_(x, mod.gate_a, self.attention(h, w, cos, sin, spec), segments)
        h = norm(x, w.norm2, self.norm_eps, mod.shift_m, mod.scale_m, segments)
        return self.ops.gate_(x, mod.gate_m, self.mlp(h, w), segments)


def rope_tables(positions: torch.Tensor, inv_freq: torch.Tensor, dtype: torch.dtype) -> Tuple[torch.Tensor, torch.Tensor]:
    """[S, 3] (t, h, w) positions -> cos, sin [S, 3 F] in `dtype` (layout.py:265-273: all t frequencies, then h, then w)."""
    ang = (positions.to(torch.float32).unsqueeze(-1) * inv_freq.to(torch.float32).view(1, 1, -1)).reshape(positions.shape[0], -1)
    return ang.cos().to(dtype), ang.sin().to(dtype)


def video_audio_positions(frames: int, h: int, w: int, audio: int, device) -> torch.Tensor:
    """Token positions of a packed video (frames x h x w patches) + audio sequence: video tokens get (t, y, x), audio
    tokens (t, 0, 0) -- the layout of the benchmark's single-stream block."""
    t = torch.arange(frames, device=device).view(-1, 1, 1).expand(frames, h, w)
    y = torch.arange(h, device=device).view(1, -1, 1).expand(frames, h, w)
    xx = torch.arange(w, device=device).view(1, 1, -1).expand(frames, h, w)
    vid = torch.stack([t, y, xx], -1).reshape(-1, 3)
    aud = torch.stack([torch.arange(audio, device=device), torch.zeros(audio, device=device, dtype=torch.long),
                       torch.zeros(audio, device=device, dtype=torch.long)], -1)
    return torch.cat([vid, aud]).to(torch.float32)
