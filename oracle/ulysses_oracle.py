"""CPU restatement of cozy-runtime's Ulysses context-parallel attention (TEST INFRASTRUCTURE ONLY).

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU legs use this module, and only as
the checker. Each function cites the reference lines it restates; paths are relative to the
cozy-runtime project root. All arithmetic is torch on CPU in fp32 or fp64.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Sequence

import torch
from torch import Tensor

E4M3_MAX = 448.0
#: attention_fp8.py:33-38: the value a head's amax maps onto, and the descale floor
E4M3_TARGET = 440.0
SCALE_FLOOR = 1e-12


def sequence_rows(total: int, world: int) -> list[int]:
    """Rows each rank holds: `torch.tensor_split` along the sequence, the first `total % world`
    ranks one row longer (src/cozy_runtime/internal/parallel/cp.py:166-174, Diffusers'
    `ulysses_anything=True`)."""
    base, extra = divmod(total, world)
    return [base + (1 if rank < extra else 0) for rank in range(world)]


def heads_padded(heads: int, world: int) -> int:
    """Heads rounded up to a multiple of the degree with zero heads
    (src/cozy_runtime/internal/parallel/ulysses.py:647)."""
    return heads + (-heads % world)


def owned_heads(heads: int, world: int, rank: int) -> range:
    """The query heads rank `rank` attends over: block `rank` of `padded/world` heads
    (ulysses.py:325-362 `_pack`, peer p takes heads `start + p*local ...`), less the padding."""
    local = heads_padded(heads, world) // world
    return range(min(rank * local, heads), min((rank + 1) * local, heads))


def attention_fp32(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    *,
    causal: bool = False,
    scale: float | None = None,
    dtype: torch.dtype = torch.float32,
) -> Tensor:
    """softmax(Q Kᵀ·scale) V over [batch, seq, heads, dim], computed in `dtype` per head.

    Restates src/cozy_runtime/internal/attention_upstream.py:109-147 (`sdpa`): torch SDPA on the
    transposed operands, causal aligned bottom-right when the query and key lengths differ
    (:106-107, :136-139). Grouped-query attention maps query head h to key head
    h // (Hq / Hkv), torch's `enable_gqa` rule. Returns `dtype`.
    """
    batch, sq, hq, dim = q.shape
    sk, hkv = k.shape[1], k.shape[2]
    if hq % hkv:
        raise ValueError("query heads must be a multiple of key heads")
    group = hq // hkv
    scale = 1.0 / math.sqrt(dim) if scale is None else scale
    out = torch.empty(batch, sq, hq, dim, dtype=dtype)
    mask = None
    if causal:
        rows = torch.arange(sq)[:, None] + (sk - sq)
        mask = torch.arange(sk)[None, :] > rows
    for b in range(batch):
        for h in range(hq):
            qh = q[b, :, h].to(dtype)
            kh = k[b, :, h // group].to(dtype)
            vh = v[b, :, h // group].to(dtype)
            s = (qh @ kh.T) * scale
            if mask is not None:
                s = s.masked_fill(mask, float("-inf"))
            p = torch.softmax(s, dim=-1)
            out[b, :, h] = p @ vh
    return out


def exchange(
    queries: Sequence[Tensor],
    keys: Sequence[Tensor],
    values: Sequence[Tensor],
    compute: Callable[[Tensor, Tensor, Tensor], Tensor],
) -> list[Tensor]:
    """The whole Ulysses exchange of W ranks, simulated in one process.

    `queries[r]` is rank r's [B, S_r, Hq, D] rows (likewise keys/values with Hkv heads). Restates
    src/cozy_runtime/internal/parallel/ulysses.py:633-766 (`_exchange`): heads padded to a
    multiple of W (:647) with zero heads (`_pack`, :335-340), rank p attending over heads
    `[p·local, (p+1)·local)` of the whole sequence (rows stacked in rank order, `_unpack`
    :420-432), `compute` on [B, S, local, D], the attended rows returned to their owners
    (`_land`, :435-457) and the padding cropped (:766). Grouped K/V heads (Hkv < Hq) cross as
    the query heads they serve, which is the reference's exchange after K/V replication.
    Returns each rank's [B, S_r, Hq, D] output.
    """
    world = len(queries)
    rows = [int(t.shape[1]) for t in queries]
    heads = int(queries[0].shape[2])
    hkv = int(keys[0].shape[2])
    group = heads // hkv
    q = torch.cat(list(queries), dim=1)
    k = torch.cat(list(keys), dim=1).repeat_interleave(group, dim=2)
    v = torch.cat(list(values), dim=1).repeat_interleave(group, dim=2)
    padded = heads_padded(heads, world)
    if padded != heads:
        pad = (0, 0, 0, padded - heads)
        q, k, v = (torch.nn.functional.pad(t, pad) for t in (q, k, v))
    local = padded // world
    attended = []
    for rank in range(world):
        part = slice(rank * local, (rank + 1) * local)
        attended.append(compute(q[:, :, part], k[:, :, part], v[:, :, part]))
    whole = torch.cat(attended, dim=2)[:, :, :heads]
    starts = [sum(rows[:r]) for r in range(world)]
    return [whole[:, s : s + n] for s, n in zip(starts, rows, strict=True)]


def exchange_group(
    query: Tensor,
    key: Tensor,
    value: Tensor,
    group,
    compute: Callable[[Tensor, Tensor, Tensor], Tensor],
) -> Tensor:
    """One rank's part of the exchange over a real process group (gloo on CPU): the reference's
    own CPU path for a layer, collectives included.

    Restates src/cozy_runtime/internal/parallel/ulysses.py:633-766 (`_exchange`) with its
    crossings: every rank's rows agreed over the group (the meeting, :89-133), heads padded to a
    multiple of W (:647), this rank's rows of each peer's `local` heads sent as one stacked
    [Q; K; V] block per peer by `all_to_all_single` (`_pack`/`_send`, :325-417), the whole
    sequence unpacked in rank order (:420-432), `compute` on [B, S, local, D], the attended
    rows sent back to their owners (`_returned`, :459-502), landed (:435-457) and cropped
    (:766). Grouped K/V heads cross replicated to the query heads they serve. Returns this
    rank's [B, S_r, H, D] output.
    """
    import torch.distributed as dist

    world, rank = dist.get_world_size(group), dist.get_rank(group)
    batch, mine, heads, dim = (int(n) for n in query.shape)
    group_size = heads // int(key.shape[2])
    counts = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(counts, torch.tensor([mine], dtype=torch.int64), group=group)
    rows = [int(c.item()) for c in counts]
    total = sum(rows)
    k = key.repeat_interleave(group_size, dim=2)
    v = value.repeat_interleave(group_size, dim=2)
    padded = heads_padded(heads, world)
    q = query
    if padded != heads:
        pad = (0, 0, 0, padded - heads)
        q, k, v = (torch.nn.functional.pad(t, pad) for t in (q, k, v))
    local = padded // world
    # send: for peer p, [3][S_r][B][local][D] of heads [p·local, (p+1)·local)
    stacked = torch.stack((q, k, v))  # [3, B, S_r, Hp, D]
    send = torch.cat([stacked[:, :, :, p * local:(p + 1) * local].permute(0, 2, 1, 3, 4)
                      .reshape(-1) for p in range(world)])
    block = 3 * batch * local * dim
    recv = torch.empty(total * block, dtype=q.dtype)
    dist.all_to_all_single(recv, send, [r * block for r in rows], [mine * block] * world,
                           group=group)
    parts, at = [], 0
    for r in rows:  # source r's rows, in rank order = sequence order
        parts.append(recv[at:at + r * block].view(3, r, batch, local, dim))
        at += r * block
    whole = torch.cat(parts, dim=1).permute(0, 2, 1, 3, 4)  # [3, B, S, local, D]
    attended = compute(whole[0], whole[1], whole[2])  # [B, S, local, D]
    starts = [sum(rows[:r]) for r in range(world)]
    back = torch.cat([attended[:, s:s + n].permute(1, 0, 2, 3).reshape(-1)
                      for s, n in zip(starts, rows, strict=True)])
    unit = batch * local * dim
    landed = torch.empty(world * mine * unit, dtype=attended.dtype)
    dist.all_to_all_single(landed, back, [mine * unit] * world, [r * unit for r in rows],
                           group=group)
    out = landed.view(world, mine, batch, local, dim).permute(2, 1, 0, 3, 4)
    return out.reshape(batch, mine, padded, dim)[:, :, :heads]


def head_norm_rope(
    x: Tensor,
    cos: Tensor,
    sin: Tensor,
    *,
    rotary: int,
    interleaved: bool,
    normalize: bool = True,
    weight: Tensor | None = None,
    offset: float = 0.0,
    eps: float = 1e-6,
    stride_channel: int = 1,
) -> Tensor:
    """Per-head RMSNorm (optional weight + offset), then RoPE on the first `rotary` channels.

    x: [B, S, H, D]; cos/sin: per token, `[S, C]` fp32 with column `col` of channel j read at
    `col * stride_channel` (the reference's `rope_tables` layout,
    src/cozy_runtime/accel/fusion/_kernels.py:497-517). Interleaved pairs channel 2i with 2i+1
    (table column i); split-half pairs j with j ± rotary/2 (column j). The law is the reference's
    own checker, src/cozy_runtime/internal/bench/kernels.py:819-850, of the fused kernel
    `head_norm_rope_kernel` (_kernels.py:177-240). Computed in fp64, returned fp64.
    """
    y = x.double()
    if normalize:
        y = y * torch.rsqrt(y.pow(2).mean(-1, keepdim=True) + eps)
        if weight is not None:
            y = y * (weight.double() + offset)
    out = y.clone()
    c, s = cos.double(), sin.double()
    for j in range(rotary):
        if interleaved:
            low, partner, col = j % 2 == 0, j ^ 1, j // 2
        else:
            half = rotary // 2
            low, partner, col = j < half, (j + half if j < half else j - half), j
        paired = -y[..., partner] if low else y[..., partner]
        cc = c[:, col * stride_channel][None, :, None]
        ss = s[:, col * stride_channel][None, :, None]
        out[..., j] = y[..., j] * cc + paired * ss
    return out


def quantise_e4m3_per_head(x: Tensor) -> tuple[Tensor, Tensor]:
    """Per-(batch, head) e4m3: descale = max(amax/440, 1e-12), x/descale clamped to ±448, cast
    round-to-nearest-even. Restates src/cozy_runtime/internal/attention_fp8.py:162-169
    (`quantise_eager`). x: [B, S, H, D]; returns (e4m3 codes, [B, H] fp32 descale)."""
    amax = x.abs().amax(dim=(1, 3)).float()
    descale = (amax / E4M3_TARGET).clamp_(min=SCALE_FLOOR)
    scaled = (x.float() / descale[:, None, :, None]).clamp_(-E4M3_MAX, E4M3_MAX)
    return scaled.to(torch.float8_e4m3fn), descale.contiguous()


def fp8_attention_law(
    queries: Sequence[Tensor],
    keys: Sequence[Tensor],
    values: Sequence[Tensor],
    *,
    causal: bool = False,
    block: int = 64,
    p_scale: float = 256.0,
    hadamard: bool = True,
    law: str = "block",
) -> Tensor:
    """The FP8 recipe of the video configuration over W ranks' rows, in fp32, returning the whole
    [B, S, H, D] output: K less its per-(batch, head) mean over the whole sequence (the shift of
    src/cozy_runtime/internal/parallel/ulysses.py:588-604); Q and K rotated by the orthonormal
    Hadamard (the reference's FA4-fp8 row, attention_upstream.py:293-317); Q and K as e4m3 with one scale per
    `block` rows × head, blocks of the whole sequence from multiples of `block`, cut at rank
    boundaries (`quantise_fp8_blocks` per block); V as e4m3 with one scale per (batch, head, channel) over the whole sequence
    (max(absmax/448, 1e-12)); P = exp(s - rowmax) · `p_scale` as e4m3; the row sum over the
    unquantised P; O = (P codes · V codes) · V scale / row sum. Grouped K/V heads as
    `attention_fp32`.

    `law="head"`: the reference's own FP8 row instead (`fa4_fp8`,
    src/cozy_runtime/internal/attention_upstream.py:293-317): Q and K rotated as the bf16
    matrix product `_hadamard` computes (`rotate_bf16`), no K mean, and Q, K and V each
    quantised per (batch, head) by `quantise_e4m3_per_head` (attention_fp8.py:162-169); the
    reference's kernel quantises P inside FlashAttention-4, so P follows this function's P law."""
    if law == "head":
        return _fp8_law_head(queries, keys, values, causal=causal, p_scale=p_scale)
    q = torch.cat(list(queries), dim=1).float()
    k = torch.cat(list(keys), dim=1).float()
    v = torch.cat(list(values), dim=1).float()
    k = k - k.mean(dim=1, keepdim=True)
    if hadamard:  # src/cozy_runtime/internal/attention_upstream.py:276-287 (`_hadamard`)
        h = hadamard_matrix(q.shape[-1])
        q, k = q @ h, k @ h
    starts = [0]
    for part in queries:
        starts.append(starts[-1] + int(part.shape[1]))

    def blocks(x: Tensor) -> Tensor:
        # blocks of `block` rows of the whole sequence from multiples of `block`, cut where one
        # rank's rows end and the next's begin
        out = torch.empty_like(x)
        edges = sorted({*range(0, starts[-1], block), *starts})
        for a, b in zip(edges[:-1], edges[1:], strict=True):
            codes, descale = quantise_fp8_blocks(x[:, a:b], b - a)
            out[:, a:b] = codes.float() * descale[:, 0][:, None, :, None]
        return out

    qd, kd = blocks(q), blocks(k)
    vamax = v.abs().amax(dim=1, keepdim=True)
    vscale = (vamax / E4M3_MAX).clamp(min=SCALE_FLOOR)
    vcodes = (v / vscale).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).float()
    return _fp8_attend(qd, kd, vcodes, vscale, causal=causal, p_scale=p_scale)


def rotate_bf16(x: Tensor) -> Tensor:
    """`x` times the orthonormal Hadamard of its head dimension as the reference's `_hadamard`
    computes it on bf16 (src/cozy_runtime/internal/attention_upstream.py:276-287): the matrix
    rounded to bf16, products summed in fp32, the result rounded to bf16."""
    h = hadamard_matrix(x.shape[-1]).to(torch.bfloat16).float()
    return (x.to(torch.bfloat16).float() @ h).to(torch.bfloat16)


def _fp8_law_head(queries, keys, values, *, causal: bool, p_scale: float) -> Tensor:
    q = rotate_bf16(torch.cat(list(queries), dim=1))
    k = rotate_bf16(torch.cat(list(keys), dim=1))
    v = torch.cat(list(values), dim=1).to(torch.bfloat16)
    (qc, qs), (kc, ks), (vc, vs) = (quantise_e4m3_per_head(t) for t in (q, k, v))
    qd = qc.float() * qs[:, None, :, None]
    kd = kc.float() * ks[:, None, :, None]
    vscale = vs[:, None, :, None].expand(v.shape[0], 1, v.shape[2], v.shape[3])
    return _fp8_attend(qd, kd, vc.float(), vscale, causal=causal, p_scale=p_scale)


def _fp8_attend(qd: Tensor, kd: Tensor, vcodes: Tensor, vscale: Tensor, *, causal: bool,
                p_scale: float) -> Tensor:
    """Attention over dequantised Q and K and V codes with their scales ([B, 1, Hkv, D]): P =
    exp(s - rowmax)·`p_scale` as e4m3, the row sum over the unquantised P."""
    batch, seq, hq, dim = qd.shape
    group = hq // kd.shape[2]
    out = torch.empty(batch, seq, hq, dim)
    mask = None
    if causal:
        mask = torch.arange(seq)[None, :] > torch.arange(seq)[:, None]
    for b in range(batch):
        for h in range(hq):
            s = (qd[b, :, h] @ kd[b, :, h // group].T) / math.sqrt(dim)
            if mask is not None:
                s = s.masked_fill(mask, float("-inf"))
            p = torch.exp(s - s.amax(dim=-1, keepdim=True)) * p_scale
            pq = p.clamp(max=E4M3_MAX).to(torch.float8_e4m3fn).float()
            o = pq @ vcodes[b, :, h // group]
            out[b, :, h] = o * vscale[b, 0, h // group] / p.sum(dim=-1, keepdim=True)
    return out


def hadamard_matrix(n: int) -> Tensor:
    """The orthonormal Sylvester Hadamard matrix of order n (a power of two), built as
    src/cozy_runtime/internal/attention_upstream.py:276-287 (`_hadamard`) builds it."""
    h = torch.ones(1, 1)
    while h.shape[0] < n:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)])
    return h / math.sqrt(n)


def quantise_fp8_blocks(x: Tensor, block: int = 64) -> tuple[Tensor, Tensor]:
    """e4m3 with one fp32 descale per `block` tokens × head: descale = max(amax/448, 1e-12) of the
    block, codes = RTNE(x/descale) clamped to ±448. This is the block form of the per-head law
    above (attention_fp8.py:162-169) at the granularity the FP8 video configuration names; a
    block covering the whole sequence with target 440 is that law exactly. x: [B, S, H, D];
    returns (codes [B, S, H, D], descale [B, ceil(S/block), H])."""
    batch, seq, heads, dim = x.shape
    blocks = -(-seq // block)
    pad = blocks * block - seq
    xf = torch.nn.functional.pad(x.float(), (0, 0, 0, 0, 0, pad))
    tiles = xf.view(batch, blocks, block, heads, dim)
    amax = tiles.abs().amax(dim=(2, 4))
    descale = (amax / E4M3_MAX).clamp_(min=SCALE_FLOOR)
    scaled = (tiles / descale[:, :, None, :, None]).clamp_(-E4M3_MAX, E4M3_MAX)
    codes = scaled.to(torch.float8_e4m3fn).view(batch, blocks * block, heads, dim)[:, :seq]
    return codes, descale


# --------------------------------------------------------------------------- the int8 wire
def _signs(order: int) -> Tensor:
    """The ±1 Sylvester matrix of `order` (turn.py:43-52 `signs`): [[H, H], [H, −H]] doubling."""
    turn = torch.ones(1, 1)
    while turn.shape[0] < order:
        turn = torch.cat([torch.cat([turn, turn], 1), torch.cat([turn, -turn], 1)])
    return turn


def turned(rows: Tensor) -> Tensor:
    """`rows` (last dimension a power of two) turned by the orthonormal Hadamard matrix, in fp32:
    (rows · H) · D^-½ with H the ±1 Sylvester matrix
    (src/cozy_runtime/internal/parallel/turn.py:54-58 `turned`)."""
    order = rows.shape[-1]
    return (rows.float() @ _signs(order)) * order**-0.5


def narrow_law(x: Tensor, shift: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """Rows of `x` less the turned `shift`, turned, as int8 scaled to each row's absmax/127
    (floor 2^-126 = bf16's smallest normal, rounded half away from zero), and those scales in
    `x`'s dtype (turn.py:60-70 `law`)."""
    t = turned(x)
    if shift is not None:
        t = t - shift
    tiny = torch.finfo(x.dtype).tiny
    scale = (t.abs().amax(-1, keepdim=True) * (1.0 / 127)).clamp(min=tiny).to(x.dtype)
    q = (t / scale.float()).clamp(-127, 127)
    return (q.sign() * (q.abs() + 0.5).floor()).to(torch.int8), scale


def narrow_law_back(values: Tensor, scale: Tensor) -> Tensor:
    """`narrow_law`'s rows back, in `scale`'s dtype (turn.py:73-77 `law_back`)."""
    order = values.shape[-1]
    summed = values.float() @ _signs(order)
    return (summed * (scale.float() * order**-0.5)).to(scale.dtype)


def _narrowed(x: Tensor, shift: Tensor | None = None) -> Tensor:
    """One crossing of the int8 wire: law there, law_back here."""
    return narrow_law_back(*narrow_law(x, shift))


def exchange_narrow(
    queries: Sequence[Tensor],
    keys: Sequence[Tensor],
    values: Sequence[Tensor],
    compute: Callable[[Tensor, Tensor, Tensor], Tensor],
) -> list[Tensor]:
    """`exchange` with the int8 wire (`narrow=True`), simulated in one process. Restates
    ulysses.py:588-604 and :704-766: K's sum over every rank's rows (fp32), divided by the total
    and turned, is the shift every rank takes off its K rows (`_Shift`); Q, K and V cross
    narrowed (`_pack` :353-362) and widen into the operands (`_unpack` :428-429); `compute`
    runs on them; its output (query dtype) crosses back narrowed (`_returned` :481-482) and
    widens into its owner's rows (`_land` :451-453). The law is row-local, so narrowing each
    rank's rows before the crossing equals narrowing them after it, as done here. bf16 rows
    throughout (the scales take the rows' dtype)."""
    world = len(queries)
    total = sum(int(t.shape[1]) for t in queries)
    summed = sum(k.sum(1, dtype=torch.float32) for k in keys)
    shift = turned(summed / total)  # [B, Hkv, D]
    qn = [_narrowed(q) for q in queries]
    kn = [_narrowed(k, shift[:, None]) for k in keys]
    vn = [_narrowed(v) for v in values]

    def narrow_out(a: Tensor, b: Tensor, c: Tensor) -> Tensor:
        return compute(a, b, c)

    outs = exchange(qn, kn, vn, narrow_out)
    return [_narrowed(o.to(queries[0].dtype)) for o in outs[:world]]
