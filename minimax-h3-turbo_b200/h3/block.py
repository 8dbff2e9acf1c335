"""One single-stream H3 DiT block driven through the W4A8 kernels, optionally token-sharded across GPUs.

Semantics of the reference block (h3turbo/h3/model.py:_block :234-242, _attention :196-228, _mlp :186-194 with
_rms / _scale_shift_ / _gate_ :64-115 and q/k norm + split-half RoPE, layout.py:norm_rope_ :329-356 in its "torch" form
:309-326): with AdaLN modulation rows per token segment (precomputed here, as the benchmark configuration states),

    h = rms(x, norm1) * (1 + sc_a) + sh_a                (bf16, in place)
    q, k, v = qlinear(h, qkv);  q, k <- rope(rms_h(q)), rope(rms_h(k));  o = sdpa(q, k, v)
    x = x + g_a * qlinear(o, out)
    h = rms(x, norm2) * (1 + sc_m) + sh_m
    x = x + g_m * qlinear(qlinear(h, fc1), fc2, input_act="swiglu")

Every linear is the W4A8 qlinear (kernels KA + KB); q/k norm + RoPE is the fused kernel of `rope.norm_rope_`; the
other norms, the modulation and attention are torch ops (attention through torch's SDPA library kernels, bf16).

Token sharding (rank r of P owns a contiguous slice of rows): every op above is token-wise except attention, which needs
all keys and values; each block therefore all-gathers K and V (bf16, [S_local, inner] each) over NCCL before the local
queries attend, and `gather_rows` assembles the final hidden states at the sequence boundary.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

from . import qlinear as ql
from .rope import norm_rope_
from .types import BlockWeights

Segment = Tuple[int, int, int]  # (first row, end row, modulation row)


def rms(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """F.rms_norm over the last dim with the weight in x.dtype (model.py:64-66)."""
    return F.rms_norm(x, (x.shape[-1],), weight if weight.dtype == x.dtype else weight.to(x.dtype), eps)


def scale_shift_(h: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, segments: Sequence[Segment]) -> torch.Tensor:
    for a, b, row in segments:
        if b > a:
            h[a:b].mul_(1.0 + scale[row].to(h.dtype)).add_(shift[row].to(h.dtype))
    return h


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


def rms_modulate(x: torch.Tensor, weight: torch.Tensor, eps: float, shift: torch.Tensor, scale: torch.Tensor,
                 segments: Sequence[Segment]) -> torch.Tensor:
    """h = scale_shift_(rms(x, weight, eps), shift, scale, segments) as one pass over x (model.py:64-66, 106-109) on the
    fused kernel for bf16/fp16 CUDA tensors (rows: ints, or int tensors of per-token rows as the reference's _pieces
    takes).  fp32 and CPU tensors take the reference's torch ops."""
    if not _kernel_rows(x):
        return scale_shift_(rms(x, weight, eps), shift, scale, segments)
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
    multiple of 512 or above 6144, ConvRot other than 256)."""
    x = pre.x
    if not (x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.shape[1] % 512 == 0 and x.shape[1] <= 6144
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
    """x[a:b] += other[a:b] * gate[row] per segment, in place (model.py:111-115): the fused kernel for bf16/fp16 CUDA
    rows (bit-identical to torch's addcmul_), the reference's torch ops otherwise."""
    if _kernel_rows(x) and other.shape == x.shape and other.dtype == x.dtype and x.stride(1) == 1 and x.stride(0) % 8 == 0 \
            and x.data_ptr() % 16 == 0:
        from .. import _lib

        m, hid = x.shape
        other, g = _aligned_rows(other), _aligned_rows(gate)
        table, n_seg, token_rows = _segment_args(segments, m, g.shape[0], x.device)
        _lib.check(_lib.lib().h3b_gate_residual(x.data_ptr(), _lib.act_code(x.dtype), x.stride(0), other.data_ptr(),
                                                other.stride(0), m, hid, g.data_ptr(), g.stride(0), g.shape[0],
                                                _lib.act_code(g.dtype), table, n_seg, _lib.ptr(token_rows),
                                                _lib.stream_ptr(x.device)), "gate_residual")
        return x
    for a, b, row in segments:
        if b > a:
            x[a:b].addcmul_(other[a:b], gate[row].to(x.dtype))
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
    the natural-log sum of exp of the scaled scores): torch's cuDNN fused kernel on CUDA, the explicit fp32 softmax
    elsewhere (the CPU ranks of the sharding tests)."""
    if q.is_cuda:
        r = torch.ops.aten._scaled_dot_product_cudnn_attention(q, k, v, None, True)
        return r[0], r[1].reshape(q.shape[:-1]).to(torch.float32)
    sc = torch.matmul(q.float(), k.float().transpose(-1, -2)) * (q.shape[-1] ** -0.5)
    lse = torch.logsumexp(sc, dim=-1)
    return torch.matmul(torch.exp(sc - lse.unsqueeze(-1)), v.float()).to(q.dtype), lse


def merge_attention(acc: Optional[torch.Tensor], acc_lse: Optional[torch.Tensor], o: torch.Tensor,
                    lse: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Combine attention over disjoint key sets: softmax weights renormalised by the log-sum-exps, in fp32."""
    if acc is None:
        return o.float(), lse
    new = torch.logaddexp(acc_lse, lse)
    acc = acc.mul_(torch.exp(acc_lse - new).unsqueeze(-1)).add_(o.float() * torch.exp(lse - new).unsqueeze(-1))
    return acc, new


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, spec: ShardSpec) -> torch.Tensor:
    """Attention of this rank's queries over every rank's keys and values, with the key/value shards passed round a
    ring of the ranks (P - 1 point-to-point steps) while the attention over the shard already here runs: the transfer
    of step s + 1 overlaps the attention of step s.  q, k, v: [S_local, H, D]; returns [S_local, H, D] in q.dtype."""
    import torch.distributed as dist

    p_, r_ = spec.world, spec.rank
    sizes = [b - a for a, b in (shard_rows(spec.total, p_, i) for i in range(p_))]
    cap = max(sizes)
    s, h, d = k.shape
    bufs = [torch.zeros(2, cap, h, d, dtype=k.dtype, device=k.device) for _ in range(2)]
    bufs[0][0, :s] = k
    bufs[0][1, :s] = v
    qh = q.transpose(0, 1).unsqueeze(0).contiguous()
    fused = q.is_cuda and q.dtype == torch.bfloat16 and d in (64, 128, 256)
    if fused:  # running output / log-sum-exp for the merge kernel, and the final [S, H * D] rows
        from .. import _lib

        acc = torch.empty(h, s, d, dtype=torch.float32, device=q.device)
        acc_lse = torch.empty(h, s, dtype=torch.float32, device=q.device)
        final = torch.empty(s, h * d, dtype=q.dtype, device=q.device)
    else:
        acc = acc_lse = None
    nxt, prv = (r_ + 1) % p_, (r_ - 1) % p_
    for step in range(p_):
        cur = bufs[step % 2]
        reqs = []
        if step < p_ - 1:
            reqs = dist.batch_isend_irecv([dist.P2POp(dist.isend, cur, nxt, group=spec.group),
                                           dist.P2POp(dist.irecv, bufs[(step + 1) % 2], prv, group=spec.group)])
        n = sizes[(r_ - step) % p_]  # the shard in `cur` came from rank r - step
        o, lse = attention_lse(qh, cur[0, :n].transpose(0, 1).unsqueeze(0), cur[1, :n].transpose(0, 1).unsqueeze(0))
        if fused:
            lse = lse.reshape(h, s).contiguous()
            if o.stride(3) != 1:
                o = o.contiguous()
            last = step == p_ - 1
            _lib.check(_lib.lib().h3b_attn_merge(acc.data_ptr(), acc_lse.data_ptr(), o.data_ptr(), o.stride(1), o.stride(2),
                                                 lse.data_ptr(), h, s, d, int(step == 0),
                                                 final.data_ptr() if last else None, h * d,
                                                 _lib.stream_ptr(q.device)), "attn_merge")
        else:
            acc, acc_lse = merge_attention(acc, acc_lse, o, lse)
        for rq in reqs:
            rq.wait()
    if fused:
        return final.view(s, h, d)
    return acc[0].transpose(0, 1).to(q.dtype)


class DiTBlock:
    """Runs H3 DiT blocks on the W4A8 kernels.  heads / head_dim / eps as in H3Config.  kv_exchange: "gather" (one
    all-gather of K and V per block, then one attention call) or "ring" (key/value shards passed round the ranks and
    overlapped with per-shard attention).  At config 5 on 8 B200s the all-gather measured faster (46.4 vs 54.4 ms per
    forward: eight smaller attention calls and their merges cost more than the hidden transfers), so it is the default."""

    def __init__(self, heads: int, head_dim: int, norm_eps: float = 1e-5, qk_norm_eps: float = 1e-5,
                 precision: str = "a8", attn_chunk: Optional[int] = None, linear=None, kv_exchange: str = "gather",
                 fuse_norm: Optional[bool] = None, kv_groups: int = 1):
        if kv_exchange not in ("ring", "gather"):
            raise ValueError(f"kv_exchange must be 'ring' or 'gather', got {kv_exchange!r}")
        if kv_groups < 1:
            raise ValueError(f"kv_groups must be >= 1, got {kv_groups}")
        self.kv_exchange = kv_exchange
        # "gather" over several ranks with kv_groups > 1: the key/value all-gather goes in head groups, all started at
        # once, and each group's attention runs as soon as its keys and values are in, while the later groups are still
        # in flight.  At config 5 on 2 B200s that measured slower than one all-gather (157.2 vs 152.5 ms per forward:
        # four smaller attention calls cost more than the hidden transfer), so the default is 1
        self.kv_groups = kv_groups
        self.heads, self.head_dim = heads, head_dim
        self.norm_eps, self.qk_norm_eps, self.precision = norm_eps, qk_norm_eps, precision
        self.attn_chunk = attn_chunk
        # the linear op: the W4A8 qlinear (default); tests of the token-sharding plumbing on CPU ranks pass a dense one
        self._linear = linear or (lambda x, w, input_act=None: ql.linear(x, w, precision=self.precision, input_act=input_act))
        self._linear_is_default = linear is None
        # RMSNorm + modulation fused into the quantiser of the qkv and fc1 linears: on for the default linear; a custom
        # linear opts in with fuse_norm=True and then receives a Prenorm for those two
        self._fuse_norm = linear is None if fuse_norm is None else fuse_norm

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
        norm_rope_(q, k, w.q_norm, w.k_norm, self.qk_norm_eps, cos, sin)
        if spec is not None and spec.world > 1 and self.kv_exchange == "ring":
            return self._linear(ring_attention(q, k, v, spec).reshape(s, inner), w.out)
        if spec is not None and spec.world > 1:  # every query needs every key and value
            groups = self.kv_groups if heads % self.kv_groups == 0 and not (self.attn_chunk and self.attn_chunk < s) else 1
            if groups > 1:
                return self._linear(self._grouped_gather_attention(q, k, v, spec, groups), w.out)
            k = gather_rows(k.reshape(s, inner).contiguous(), spec).view(-1, heads, hd)
            v = gather_rows(v.reshape(s, inner).contiguous(), spec).view(-1, heads, hd)
        qh = q.transpose(0, 1).unsqueeze(0)
        kh, vh = (t.transpose(0, 1).unsqueeze(0) for t in (k, v))
        step = self.attn_chunk or s
        if step >= s:
            o = F.scaled_dot_product_attention(qh, kh, vh).transpose(1, 2).reshape(s, inner)
        else:  # query rows are independent (chunks may pick another attention kernel: not bit-identical)
            o = torch.empty(s, inner, dtype=h.dtype, device=h.device)
            for a in range(0, s, step):
                o[a:a + step] = F.scaled_dot_product_attention(qh[:, :, a:a + step], kh, vh)[0].transpose(0, 1).reshape(-1, inner)
        return self._linear(o, w.out)

    def _grouped_gather_attention(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, spec: ShardSpec,
                                  groups: int) -> torch.Tensor:
        """Attention of the local queries over all ranks' keys and values, gathered in `groups` head groups: every
        group's K and V all-gathers are started first, then each group's attention waits only for its own."""
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
            qh = q[:, h0:h0 + hg].transpose(0, 1).unsqueeze(0)
            kh, vh = (t.transpose(0, 1).unsqueeze(0) for t in (kg, vg))
            o[:, h0 * hd:(h0 + hg) * hd] = F.scaled_dot_product_attention(qh, kh, vh)[0].transpose(0, 1).reshape(s, hg * hd)
        return o

    def mlp(self, h: torch.Tensor, w: BlockWeights) -> torch.Tensor:
        return self._linear(self._in_linear(h, w.fc1), w.fc2, input_act="swiglu")

    def __call__(self, x: torch.Tensor, w: BlockWeights, mod: Modulation, segments: Sequence[Segment], cos: torch.Tensor,
                 sin: torch.Tensor, spec: Optional[ShardSpec] = None) -> torch.Tensor:
        """x: [S_local, hidden] residual stream (updated in place and returned); cos/sin: [S_local, half] for these rows."""
        norm = Prenorm if self._fuse_norm else rms_modulate
        h = norm(x, w.norm1, self.norm_eps, mod.shift_a, mod.scale_a, segments)
        gate_(x, mod.gate_a, self.attention(h, w, cos, sin, spec), segments)
        h = norm(x, w.norm2, self.norm_eps, mod.shift_m, mod.scale_m, segments)
        return gate_(x, mod.gate_m, self.mlp(h, w), segments)


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
