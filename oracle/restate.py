"""CPU restatement of Drama3-Studio's quantized routed-expert hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports, links or
executes this module; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only
as the checker (or as the timed CPU port). Plain numpy, float32 IEEE arithmetic
with explicit rounding points, so every integer/byte result (FP8 bytes, route
indices, permutations) is bit-exact and every floating-point result is
reproducible on any host.

Each function cites the reference file:line it restates (paths relative to the
Drama3-Studio source tree):

* ``route_topk``         - ``src/drama_low_vram/backbone_graph.py:317-323``
                            (softmax(gate.float()) -> topk -> renorm -> cast),
                            with torch's CUDA softmax / topk tie order restated.
* ``permute_routes``     - ``src/drama_low_vram/offload.py:1206-1211``
                            (stable argsort + bincount over flat route IDs).
* ``dequantize_fp8_blocks`` / ``fp8_dequant_pairs`` / ``fp8_dequant_forward``
                          - ``src/drama_low_vram/offload.py:44-56, 202-244``
                            (TorchExpertBackend, the PyTorch W16A16 dequant path).
* ``quantize_fp8_activations`` / ``w8a8_pairs``
                          - ``src/drama_low_vram/fp8_cpu_reference.py:14-52`` and
                            ``native/src/runtime.cpp:162-237``,
                            ``native/src/fp8_reference.cpp:10-93`` (official W8A8
                            blockwise contract).
* ``int4_dequant_pairs`` / ``int4_forward``
                          - ``src/drama_low_vram/quantized_kernels.py:48-112, 217-248``
                            (mode 0 GPTQ W4A16), extended with explicit uint4
                            zero-points (``zp = 8`` reproduces the reference).
* ``convrot_rotate`` / ``quantize_rows_int8`` / ``convrot_grid`` /
  ``convrot_pairs`` / ``convrot_forward``
                          - ``src/drama_low_vram/quantized_kernels.py:15-45, 115-189,
                            217-248`` (W8A8 modes 1-3: INT8-ConvRot, W6A8, W4A8
                            codebook; layouts of ``quantized_model.py:45-68, 114-151``).
* ``shared_expert`` / ``post_moe``
                          - ``src/drama_low_vram/backbone_graph.py:327-337`` (shared
                            expert, sigmoid gate, ``after_mixer + (experts + shared)``).
* ``rms_norm`` / ``stack_layer`` - the decode layer of
                            ``src/drama_low_vram/backbone_graph.py:306-337`` without
                            the mixer and the shared expert.

Pinning: ``tests/golden/`` holds vectors produced by the reference's own Python
code (imported in the build container) and by the reference's router ops run on
a B200; ``tests/test_oracle.py`` checks this module against every one of them,
and against the reference's native C++ executor built from source under
``oracle/_ref``.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
FP8_BLOCK = 128
FP8_MAX = 448.0

# --------------------------------------------------------------------------
# Scalar formats
# --------------------------------------------------------------------------


def bf16_bits(x) -> np.ndarray:
    """float32 -> bf16 bit patterns, round-to-nearest-even, NaN kept."""
    x = np.asarray(x, dtype=F32)
    bits = x.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = np.where(nan, (bits >> 16).astype(np.uint16) | np.uint16(0x40), rounded)
    return rounded


def from_bf16_bits(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


def round_bf16(x) -> np.ndarray:
    """Round float32 values to bf16 and return them as float32."""
    return from_bf16_bits(bf16_bits(x))


def round_to(x, dtype: str) -> np.ndarray:
    """Round float32 values to the compute dtype of the reference's tensors."""
    x = np.asarray(x, dtype=F32)
    if dtype == "bfloat16":
        return round_bf16(x)
    if dtype == "float16":
        return x.astype(np.float16).astype(F32)
    if dtype == "float32":
        return x
    raise ValueError(f"unsupported dtype {dtype}")


def _fp8_table() -> np.ndarray:
    # native/src/fp8_reference.cpp:10-17 (E4M3FN: bias 7, 0x7f/0xff are NaN).
    table = np.empty(256, dtype=F32)
    for value in range(256):
        mag, exp, man = value & 127, (value & 127) >> 3, value & 7
        if mag == 127:
            result = np.nan
        elif exp == 0:
            result = man * 2.0 ** -9
        else:
            result = (1.0 + man / 8.0) * 2.0 ** (exp - 7)
        table[value] = -result if value & 128 else result
    return table


FP8_TABLE = _fp8_table()


def decode_fp8(raw) -> np.ndarray:
    return FP8_TABLE[np.asarray(raw, dtype=np.uint8)]


def encode_fp8(values) -> np.ndarray:
    """float32 -> E4M3FN bytes, RNE, saturating at 448 (fp8_reference.cpp:19-36)."""
    v = np.asarray(values, dtype=F32)
    if not np.isfinite(v).all():
        raise ValueError("Non-finite FP8 input")
    sign = np.where(np.signbit(v), np.uint8(128), np.uint8(0))
    a = np.minimum(np.abs(v), F32(FP8_MAX))
    # Subnormal range: multiples of 2^-9, round half to even.
    scaled = a * F32(512.0)
    whole = np.floor(scaled)
    frac = scaled - whole
    whole_i = whole.astype(np.int64)
    up = (frac > 0.5) | ((frac == 0.5) & (whole_i & 1 == 1))
    sub = (whole_i + up).astype(np.uint32)
    # Normal range: round the float32 mantissa to 3 bits.
    bits = a.view(np.uint32).astype(np.uint64)
    bits = bits + (1 << 19) - 1 + ((bits >> 20) & 1)
    normal = ((bits >> 20) - (120 << 3)).astype(np.int64)
    normal = np.clip(normal, 0, 255).astype(np.uint32)
    code = np.where(a < F32(0.015625), sub, normal).astype(np.uint8)
    return (code | sign).astype(np.uint8)


# --------------------------------------------------------------------------
# Router: softmax -> top-k -> renormalise -> cast (backbone_graph.py:317-323)
# --------------------------------------------------------------------------


def _warp_butterfly_sum(values: np.ndarray) -> np.ndarray:
    """Sum the last axis (32 lanes) the way a shfl_xor butterfly does."""
    v = values.astype(F32).copy()
    lanes = v.shape[-1]
    offset = lanes // 2
    idx = np.arange(lanes)
    while offset:
        v = (v + v[..., idx ^ offset]).astype(F32)
        offset //= 2
    return v[..., 0]


def softmax_rows(logits) -> np.ndarray:
    """fp32 softmax over the last axis in torch's persistent-warp order.

    torch's CUDA softmax for rows of <= 1024 fp32 values keeps one row per warp:
    lane ``l`` holds elements ``l + 32*i``, adds its ``exp(x - max)`` terms in
    ``i`` order, then the warp adds lane sums with a xor butterfly; each output
    is ``exp(x - max) / sum``.
    """
    x = np.asarray(logits, dtype=F32)
    rows, width = x.shape
    p2 = 1 << max(0, (width - 1).bit_length())
    lanes = min(p2, 32)
    iters = p2 // lanes
    padded = np.full((rows, iters * lanes), -np.inf, dtype=F32)
    padded[:, :width] = x
    m = padded.max(axis=1, keepdims=True)
    with np.errstate(invalid="ignore"):
        e = np.exp((padded - m).astype(F32)).astype(F32)
    e[:, width:] = 0
    lane_sums = np.zeros((rows, lanes), dtype=F32)
    by_iter = e.reshape(rows, iters, lanes)
    for i in range(iters):
        lane_sums = (lane_sums + by_iter[:, i, :]).astype(F32)
    total = _warp_butterfly_sum(lane_sums)
    return (e[:, :width] / total[:, None]).astype(F32)


def _bitonic_sort_desc(keys: np.ndarray, vals: np.ndarray, count: int):
    """Restates torch's 32-slot key/value bitonic network (SmallBitonicSort).

    Positions ``count..31`` are invalid padding that always sinks to the end;
    the comparator is ``a > b`` (descending). Ties are resolved by the network,
    not by index: this is what ``topk(sorted=True)`` returns on CUDA for k<=32.
    """
    n = 32
    k = np.zeros(keys.shape[:-1] + (n,), dtype=F32)
    v = np.zeros(vals.shape[:-1] + (n,), dtype=np.int64)
    ok = np.zeros(keys.shape[:-1] + (n,), dtype=bool)
    k[..., :count] = keys
    v[..., :count] = vals
    ok[..., :count] = True

    def stage(stride: int, flags: np.ndarray) -> None:
        t = np.arange(n // 2)
        pos = 2 * t - (t & (stride - 1))
        a, b = pos, pos + stride
        ka, kb = k[..., a], k[..., b]
        va, vb = v[..., a], v[..., b]
        oka, okb = ok[..., a], ok[..., b]
        swap = ((ka > kb) & oka) | ~okb
        do = swap == flags
        k[..., a], k[..., b] = np.where(do, kb, ka), np.where(do, ka, kb)
        v[..., a], v[..., b] = np.where(do, vb, va), np.where(do, va, vb)
        ok[..., a], ok[..., b] = np.where(do, okb, oka), np.where(do, oka, okb)

    size = 2
    t = np.arange(n // 2)
    while size < n:
        flags = (t & (size // 2)) != 0
        stride = size // 2
        while stride:
            stage(stride, flags)
            stride //= 2
        size *= 2
    stride = n // 2
    while stride:
        stage(stride, np.zeros(n // 2, dtype=bool))
        stride //= 2
    return k[..., :count], v[..., :count]


def topk_rows(probs: np.ndarray, top_k: int):
    """torch.topk(largest=True, sorted=True) as its CUDA kernel orders results.

    Selection (gatherTopK): every value strictly greater than the k-th largest,
    in index order, then values equal to it in index order until k are taken.
    Ordering: the 32-slot bitonic network above (k <= 32).
    """
    if not 1 <= top_k <= 32:
        raise ValueError("top_k must be in [1, 32]")
    p = np.asarray(probs, dtype=F32)
    rows, width = p.shape
    kth = -np.sort(-p, axis=1)[:, top_k - 1]
    keys = np.zeros((rows, top_k), dtype=F32)
    idx = np.zeros((rows, top_k), dtype=np.int64)
    for r in range(rows):
        greater = np.nonzero(p[r] > kth[r])[0]
        equal = np.nonzero(p[r] == kth[r])[0][: top_k - greater.size]
        chosen = np.concatenate([greater, equal])
        keys[r] = p[r, chosen]
        idx[r] = chosen
    return _bitonic_sort_desc(keys, idx, top_k)


def _pairwise_tree_sum(values: np.ndarray) -> np.ndarray:
    """Sum the last axis as shfl_down steps 1, 2, 4, ... combine lanes."""
    v = values.astype(F32).copy()
    width = v.shape[-1]
    p2 = 1 << max(0, (width - 1).bit_length())
    if p2 != width:
        pad = np.zeros(v.shape[:-1] + (p2 - width,), dtype=F32)
        v = np.concatenate([v, pad], axis=-1)
    step = 1
    while step < p2:
        v[..., 0:p2:2 * step] = (v[..., 0:p2:2 * step] + v[..., step:p2:2 * step]).astype(F32)
        step *= 2
    return v[..., 0]


def route_topk(logits, top_k: int = 8, renormalize: bool = True,
               out_dtype: str = "bfloat16"):
    """backbone_graph.py:319-323 on fp32 copies of the gate logits.

    Returns (ids int64 [T,k], weights float32 [T,k] holding ``out_dtype``
    values, probabilities float32 [T,E]).
    """
    probs = softmax_rows(logits)
    values, ids = topk_rows(probs, top_k)
    if renormalize:
        total = _pairwise_tree_sum(values)
        values = (values / total[:, None]).astype(F32)
    return ids, round_to(values, out_dtype), probs


# --------------------------------------------------------------------------
# Gather / permute (offload.py:1206-1211)
# --------------------------------------------------------------------------


def permute_routes(flat_ids, num_experts: int):
    """Stable argsort of route IDs plus per-expert counts and start offsets."""
    ids = np.asarray(flat_ids, dtype=np.int64).reshape(-1)
    if ids.size and (ids.min() < 0 or ids.max() >= num_experts):
        raise ValueError("route id outside [0, experts)")
    order = np.argsort(ids, kind="stable").astype(np.int64)
    counts = np.bincount(ids, minlength=num_experts).astype(np.int64)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    return order, counts, offsets


# --------------------------------------------------------------------------
# FP8 128x128 block weights
# --------------------------------------------------------------------------


def quantize_weight_blocks(weight):
    """Synthetic bank builder: per 128x128 block scale = amax/448, RNE E4M3.

    Not a reference function: BASELINE's generator ("N(0,0.02) values before
    quantisation, fp32 scale per 128x128 block"). Returns (bytes, scales).
    """
    w = np.asarray(weight, dtype=F32)
    *lead, rows, cols = w.shape
    rb, cb = rows // FP8_BLOCK, cols // FP8_BLOCK
    blocks = w.reshape(*lead, rb, FP8_BLOCK, cb, FP8_BLOCK)
    amax = np.abs(blocks).max(axis=(-3, -1))
    scale = np.maximum(amax, F32(1e-12)).astype(F32) / F32(FP8_MAX)
    scale = scale.astype(F32)
    q = encode_fp8(blocks / scale[..., :, None, :, None])
    return q.reshape(w.shape), scale


def dequantize_fp8_blocks(raw, scale, dtype: str = "bfloat16") -> np.ndarray:
    """offload.py:44-56: (fp8 -> fp32) * block scale, rounded to ``dtype``."""
    raw = np.asarray(raw, dtype=np.uint8)
    rows, cols = raw.shape[-2:]
    rb, cb = np.asarray(scale).shape[-2:]
    if rows != rb * FP8_BLOCK or cols != cb * FP8_BLOCK:
        raise ValueError("FP8 weight shape does not match its 128x128 block scales")
    lead = raw.shape[:-2]
    blocks = decode_fp8(raw).reshape(*lead, rb, FP8_BLOCK, cb, FP8_BLOCK)
    scaled = (blocks * np.asarray(scale, dtype=F32)[..., :, None, :, None]).astype(F32)
    return round_to(scaled.reshape(raw.shape), dtype)


def silu(x) -> np.ndarray:
    x = np.asarray(x, dtype=F32)
    with np.errstate(over="ignore"):
        return (x / (F32(1.0) + np.exp(-x).astype(F32))).astype(F32)


def _ffn_pair(x_row, w13, w2, dtype: str):
    """One routed pair of the W16A16 dequant path, before route weighting.

    offload.py:237-238: ``gate, up = F.linear(x, W13).chunk(2)``;
    ``F.linear(F.silu(gate) * up, W2)`` with every op in ``dtype``.
    """
    inter = w13.shape[0] // 2
    gu = round_to(np.asarray(x_row, dtype=F32) @ w13.T, dtype)
    gate, up = gu[:inter], gu[inter:]
    act = round_to(round_to(silu(gate), dtype) * up, dtype)
    return round_to(act @ w2.T, dtype)


def fp8_dequant_pairs(x, ids, weights, bank, dtype: str = "bfloat16"):
    """TorchExpertBackend.forward_pairs (offload.py:215-244): fp32 [P,H].

    ``bank`` is a dict with w13_weight (uint8 [S,2I,H]), w13_scale_inv
    ([S,2I/128,H/128] f32), w2_weight, w2_scale_inv; ``x`` holds ``dtype``
    values as float32; ``weights`` holds route weights as float32.
    """
    x = np.asarray(x, dtype=F32)
    ids = np.asarray(ids, dtype=np.int64).reshape(-1)
    weights = np.asarray(weights, dtype=F32).reshape(-1)
    out = np.empty((ids.size, x.shape[1]), dtype=F32)
    cache: dict[int, tuple[np.ndarray, np.ndarray]] = {}
    for row, slot in enumerate(ids.tolist()):
        if slot not in cache:
            cache[slot] = (
                dequantize_fp8_blocks(bank["w13_weight"][slot], bank["w13_scale_inv"][slot], dtype),
                dequantize_fp8_blocks(bank["w2_weight"][slot], bank["w2_scale_inv"][slot], dtype),
            )
        w13, w2 = cache[slot]
        out[row] = (_ffn_pair(x[row], w13, w2, dtype) * weights[row]).astype(F32)
    return out


def combine_slots(pairs, tokens: int, top_k: int, dtype: str) -> np.ndarray:
    """offload.py:212 / 1244: fp32 sum over route slots in slot order, cast."""
    p = np.asarray(pairs, dtype=F32).reshape(tokens, top_k, -1)
    acc = np.zeros((tokens, p.shape[-1]), dtype=F32)
    for slot in range(top_k):
        acc = (acc + p[:, slot]).astype(F32)
    return round_to(acc, dtype)


def fp8_dequant_forward(x, ids, weights, bank, dtype: str = "bfloat16"):
    """TorchExpertBackend.forward (offload.py:202-213): [T,H] in ``dtype``."""
    x = np.asarray(x, dtype=F32)
    tokens, top_k = np.asarray(ids).shape
    pairs = fp8_dequant_pairs(np.repeat(x, top_k, axis=0), np.asarray(ids).reshape(-1),
                              np.asarray(weights).reshape(-1), bank, dtype)
    return combine_slots(pairs, tokens, top_k, dtype)


# --------------------------------------------------------------------------
# Official W8A8 blockwise contract (fp8_cpu_reference.py, native runtime.cpp)
# --------------------------------------------------------------------------


def quantize_fp8_activations(values):
    """1x128 activation quantisation: scale = max(amax,1e-10) * (1/448).

    fp8_cpu_reference.py:14-20; fp8_reference.cpp:52-93. Returns (bytes, scales).
    """
    v = np.asarray(values, dtype=F32).reshape(-1, FP8_BLOCK)
    if not np.isfinite(v).all():
        raise ValueError("Non-finite activation")
    amax = np.maximum(np.abs(v).max(axis=1), F32(1e-10)).astype(F32)
    scales = (amax * F32(1.0 / 448.0)).astype(F32)
    q = encode_fp8((v / scales[:, None]).astype(F32))
    return q.reshape(np.asarray(values).shape), scales


def _w8a8_rows(raw, scale, q, qs):
    """runtime.cpp:162-172: per 128 block, sequential fp32 dot, then
    ``acc = fma(dot * sa, sb, acc)`` (fma emulated exactly in float64)."""
    rows, cols = raw.shape
    w = decode_fp8(raw).reshape(rows, cols // FP8_BLOCK, FP8_BLOCK)
    a = decode_fp8(q).reshape(cols // FP8_BLOCK, FP8_BLOCK)
    acc = np.zeros(rows, dtype=F32)
    for block in range(cols // FP8_BLOCK):
        dot = np.zeros(rows, dtype=F32)
        prod = (w[:, block, :] * a[block][None, :]).astype(F32)
        for k in range(FP8_BLOCK):
            dot = (dot + prod[:, k]).astype(F32)
        scaled = (dot * qs[block]).astype(F32)
        sb = np.repeat(scale[:, block], FP8_BLOCK)[:rows].astype(np.float64)
        acc = (scaled.astype(np.float64) * sb + acc.astype(np.float64)).astype(F32)
    return acc


def w8a8_pairs(x_row, ids, weights, bank):
    """Ordered weighted fp32 partials of one bf16 row (runtime.cpp:173-237)."""
    x = np.asarray(x_row, dtype=F32).reshape(-1)
    q, qs = quantize_fp8_activations(x)
    out = []
    for slot, route_weight in zip(np.asarray(ids).reshape(-1).tolist(),
                                  np.asarray(weights, dtype=F32).reshape(-1).tolist()):
        gu = _w8a8_rows(bank["w13_weight"][slot], bank["w13_scale_inv"][slot], q, qs)
        inter = gu.size // 2
        gu = round_bf16(gu)
        gate, up = gu[:inter], gu[inter:]
        hidden = ((gate / (F32(1.0) + np.exp(-gate).astype(F32))).astype(F32) * up).astype(F32)
        hq, hs = quantize_fp8_activations(hidden)
        down = _w8a8_rows(bank["w2_weight"][slot], bank["w2_scale_inv"][slot], hq, hs)
        out.append((down * F32(route_weight)).astype(F32))
    return np.stack(out)


# --------------------------------------------------------------------------
# INT4 W4A16 (quantized_kernels.py mode 0), asymmetric extension
# --------------------------------------------------------------------------


def unpack_int4(words, k: int) -> np.ndarray:
    """[.., K/8] int32 -> [.., K] codes; nibble k%8 at bit 4*(k%8)
    (quantized_kernels.py:79-80)."""
    w = np.asarray(words).astype(np.int64) & 0xFFFFFFFF
    shifts = np.arange(8, dtype=np.int64) * 4
    codes = (w[..., None] >> shifts) & 15
    return codes.reshape(*w.shape[:-1], k).astype(np.int64)


def pack_int4(codes) -> np.ndarray:
    """Inverse of ``unpack_int4`` (tests/test_quantized_kernels.py:8-12)."""
    c = np.asarray(codes, dtype=np.int64)
    k = c.shape[-1]
    c = c.reshape(*c.shape[:-1], k // 8, 8)
    words = np.zeros(c.shape[:-1], dtype=np.int64)
    for shift in range(8):
        words |= (c[..., shift] & 15) << (4 * shift)
    return words.astype(np.uint32).view(np.int32)


def unpack_zeros(qzeros, rows: int) -> np.ndarray:
    """[N/8, G] int32 (8 row zero-points per word, row%8 nibble) -> [N, G]."""
    z = np.asarray(qzeros).astype(np.int64) & 0xFFFFFFFF
    shifts = np.arange(8, dtype=np.int64) * 4
    codes = (z[:, None, :] >> shifts[None, :, None]) & 15
    return codes.reshape(rows, z.shape[1]).astype(np.int64)


def pack_zeros(zeros) -> np.ndarray:
    z = np.asarray(zeros, dtype=np.int64)
    rows, groups = z.shape
    z = z.reshape(rows // 8, 8, groups)
    words = np.zeros((rows // 8, groups), dtype=np.int64)
    for shift in range(8):
        words |= (z[:, shift, :] & 15) << (4 * shift)
    return words.astype(np.uint32).view(np.int32)


def dequantize_int4(words, scales, qzeros, k: int, dtype: str = "bfloat16"):
    """quantized_kernels.py:78-81: ((code - zp) * scale).to(dtype), group 128.

    ``qzeros`` None means the reference's implicit zero-point 8.
    """
    codes = unpack_int4(words, k)
    rows = codes.shape[0]
    zp = np.full((rows, k // 128), 8, dtype=np.int64) if qzeros is None else unpack_zeros(qzeros, rows)
    scale = np.asarray(scales, dtype=F32)
    level = (codes - np.repeat(zp, 128, axis=1)).astype(F32)
    return round_to((level * np.repeat(scale, 128, axis=1)).astype(F32), dtype)


def int4_dequant_pairs(x, ids, weights, bank, dtype: str = "bfloat16"):
    """QuantizedExpertBackend._pairs (quantized_kernels.py:231-245), fp32 [P,H].

    projection_torch multiplies in fp32 (line 106) and rounds each projection
    to bf16 (line 111) before weighting.
    """
    x = np.asarray(x, dtype=F32)
    ids = np.asarray(ids, dtype=np.int64).reshape(-1)
    weights = np.asarray(weights, dtype=F32).reshape(-1)
    hidden = x.shape[1]
    inter = bank["w2_weight"].shape[2] * 8
    out = np.empty((ids.size, hidden), dtype=F32)
    cache: dict[int, tuple[np.ndarray, np.ndarray]] = {}
    for row, slot in enumerate(ids.tolist()):
        if slot not in cache:
            z13 = None if bank.get("w13_qzeros") is None else bank["w13_qzeros"][slot]
            z2 = None if bank.get("w2_qzeros") is None else bank["w2_qzeros"][slot]
            cache[slot] = (
                dequantize_int4(bank["w13_weight"][slot], bank["w13_scale_inv"][slot], z13, hidden, dtype),
                dequantize_int4(bank["w2_weight"][slot], bank["w2_scale_inv"][slot], z2, inter, dtype),
            )
        w13, w2 = cache[slot]
        gu = round_bf16(x[row] @ w13.T)
        gu = round_to(gu, dtype)
        gate, up = gu[:inter], gu[inter:]
        act = round_to(round_to(silu(gate), dtype) * up, dtype)
        down = round_bf16(act @ w2.T)
        out[row] = (down * weights[row]).astype(F32)
    return out


def int4_forward(x, ids, weights, bank, dtype: str = "bfloat16"):
    """QuantizedExpertBackend.forward (quantized_kernels.py:222-229)."""
    x = np.asarray(x, dtype=F32)
    tokens, top_k = np.asarray(ids).shape
    pairs = int4_dequant_pairs(np.repeat(x, top_k, axis=0), np.asarray(ids).reshape(-1),
                               np.asarray(weights).reshape(-1), bank, dtype)
    return combine_slots(pairs, tokens, top_k, dtype)


# --------------------------------------------------------------------------
# Decode stack layer (backbone_graph.py:306-337 without mixer / shared expert)
# --------------------------------------------------------------------------

NORM_THREADS = 256  # the fused router kernel's reduction geometry


def rms_norm(hidden, gamma, eps: float = 1e-6) -> np.ndarray:
    """bf16(x * (1/sqrt(mean(x^2) + eps)) * gamma), fixed fp32 reduction order.

    Order (shared with the CUDA router kernel): 256 threads each add the squares
    of ``H/256`` consecutive elements in order; 32-lane xor butterflies; the 8
    warp totals are added in warp order. mean = sum * (1/H).
    """
    x = np.asarray(hidden, dtype=F32)
    rows, width = x.shape
    per = width // NORM_THREADS
    sq = (x * x).astype(F32).reshape(rows, NORM_THREADS, per)
    thread = np.zeros((rows, NORM_THREADS), dtype=F32)
    for i in range(per):
        thread = (thread + sq[:, :, i]).astype(F32)
    warps = _warp_butterfly_sum(thread.reshape(rows, NORM_THREADS // 32, 32))
    total = np.zeros(rows, dtype=F32)
    for w in range(NORM_THREADS // 32):
        total = (total + warps[:, w]).astype(F32)
    mean = (total * F32(1.0 / width)).astype(F32)
    inv = (F32(1.0) / np.sqrt((mean + F32(eps)).astype(F32))).astype(F32)
    y = ((x * inv[:, None]).astype(F32) * np.asarray(gamma, dtype=F32)[None, :]).astype(F32)
    return round_bf16(y)


GATE_LANES = 32


def gate_logits(normed, gate_weight) -> np.ndarray:
    """bf16 logits of the bf16 gate GEMV, fixed fp32 order.

    Order (shared with the CUDA router kernel): lane ``l`` owns elements
    ``256*i + 8*l + j`` (i over H/256, j over 8), adds ``x*w`` products in
    (i, j) order with separate multiply and add; lanes combine by a xor
    butterfly. Result rounded to bf16 like ``F.linear`` in bf16.
    """
    x = np.asarray(normed, dtype=F32)
    g = np.asarray(gate_weight, dtype=F32)
    rows, width = x.shape
    experts = g.shape[0]
    chunks = width // 256
    xr = x.reshape(rows, chunks, GATE_LANES, 8)
    gr = g.reshape(experts, chunks, GATE_LANES, 8)
    acc = np.zeros((rows, experts, GATE_LANES), dtype=F32)
    for i in range(chunks):
        for j in range(8):
            prod = (xr[:, None, i, :, j] * gr[None, :, i, :, j]).astype(F32)
            acc = (acc + prod).astype(F32)
    return round_bf16(_warp_butterfly_sum(acc))


def stack_layer(hidden, gamma, gate_weight, bank, top_k: int = 8, eps: float = 1e-6):
    """One layer: h + experts(norm(h)) with routing, all bf16 boundaries.

    Returns (new_hidden, normed, ids, weights).
    """
    h = np.asarray(hidden, dtype=F32)
    normed = rms_norm(h, gamma, eps)
    logits = gate_logits(normed, gate_weight)
    ids, weights, _ = route_topk(logits, top_k, True, "bfloat16")
    moe = fp8_dequant_forward(normed, ids, weights, bank, "bfloat16")
    return round_bf16(h + moe), normed, ids, weights


# --------------------------------------------------------------------------
# W8A8 modes 1-3 (quantized_kernels.py:15-45, 115-189, 217-248)
# --------------------------------------------------------------------------

# The regular H4 basis whose 4-fold Kronecker power, divided by 16, rotates
# each 256-column group of the activations (quantized_kernels.py:30-45). It is
# symmetric, so x @ M equals M @ x.
H4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64)
CONVROT_GROUP = 256


def round_from_f64(values, dtype: str) -> np.ndarray:
    """One round-to-nearest-even from float64 to ``dtype`` (returned as float32)."""
    v = np.asarray(values, dtype=np.float64)
    if dtype == "float32":
        return v.astype(F32)
    digits, min_exp = {"bfloat16": (8, -133), "float16": (11, -24)}[dtype]
    _, exp = np.frexp(v)
    ulp = np.ldexp(1.0, np.maximum(exp - digits, min_exp))
    return (np.round(v / ulp) * ulp).astype(F32)


def convrot_rotate(x, dtype: str = "bfloat16") -> np.ndarray:
    """``x.reshape(-1, 256) @ H`` rounded to ``dtype`` (quantized_kernels.py:40, 65).

    Computed as four radix-4 stages in float64 (stage s transforms base-4 digit
    s, least significant first; each output adds its four inputs in digit
    order), then divided by 16 and rounded once. For bf16/f16 inputs the sums
    are exact whenever a row's magnitudes span fewer than ~2^37, so this is the
    correctly rounded product; the reference's bf16 matmul accumulates in fp32
    and differs only where that accumulation rounds across a bf16 boundary.
    The sm_100a kernel runs the same stages in the same order.
    """
    x = np.asarray(x, dtype=np.float64)
    rows, k = x.shape
    if k % CONVROT_GROUP:
        raise ValueError("ConvRot rows need a multiple of 256 columns")
    y = x.reshape(rows, k // CONVROT_GROUP, 4, 4, 4, 4)  # digits 3, 2, 1, 0
    for axis in (5, 4, 3, 2):  # digit 0 first
        moved = np.moveaxis(y, axis, -1)
        out = np.empty_like(moved)
        for d in range(4):
            acc = moved[..., 0] * H4[0, d]
            for i in range(1, 4):
                acc = acc + moved[..., i] * H4[i, d]
            out[..., d] = acc
        y = np.moveaxis(out, -1, axis)
    return round_from_f64(y.reshape(rows, k) / 16.0, dtype)


def quantize_rows_int8(rotated):
    """Per-row symmetric INT8 (``_row_quant``, quantized_kernels.py:15-23;
    ``projection_torch`` 66-67): scale = max(amax, 1e-12) / 127, q = rint(x / scale)
    clamped to +-127, all in IEEE fp32. Returns (q int8 [R,K], scale fp32 [R])."""
    r = np.asarray(rotated, dtype=F32)
    amax = np.abs(r).max(axis=1)
    scale = (np.maximum(amax, F32(1e-12)) / F32(127.0)).astype(F32)
    q = np.rint((r / scale[:, None]).astype(F32))
    return np.clip(q, -127, 127).astype(np.int8), scale


def convrot_grid(weight, scales, mode: int, k: int):
    """One expert's int8 weight grid [N, K] and per-row channel scale [N]
    (``_quant_gemm`` MODE 1-3, quantized_kernels.py:139-170; layouts of
    quantized_model.py:45-68, 114-151).

    mode 1: int8 weights, fp32 scale [N, 1].
    mode 2: K/2 bytes of low nibbles (column 2j in the low nibble of byte j),
            then K/4 bytes of top-two bits (column 4j+i at bits 2i of byte j);
            level = code - 32.
    mode 3: K/2 bytes of 4-bit codes; level = codebook[code], the 16 fp32
            codebook entries stored in bytes K/16+4..K/16+8 of rows 0..15.
    modes 2/3: per-16-column FP8 E4M3 relative scales in scale bytes [0, K/16),
            the fp32 channel scale in bytes [K/16, K/16+4);
            grid = clamp(rint(level * relative), +-127) in fp32.
    """
    w = np.asarray(weight)
    s = np.asarray(scales)
    if mode == 1:
        return w.astype(np.int8), s.reshape(-1).astype(F32)
    raw = w.view(np.uint8).astype(np.int64)
    n = raw.shape[0]
    low = raw[:, :k // 2]
    code = np.stack((low & 15, low >> 4), axis=-1).reshape(n, k)
    aux = s.view(np.uint8)
    if mode == 2:
        high = raw[:, k // 2:k // 2 + k // 4]
        top = (high[..., None] >> (np.arange(4) * 2)) & 3
        code = code | (top.reshape(n, k) << 4)
        level = (code - 32).astype(F32)
    elif mode == 3:
        table = np.ascontiguousarray(aux[:16, k // 16 + 4:k // 16 + 8]).view(F32).reshape(16)
        level = table[code]
    else:
        raise ValueError(f"unsupported W8A8 mode {mode}")
    relative = decode_fp8(aux[:, :k // 16]).astype(F32)
    grid = np.rint((level * np.repeat(relative, 16, axis=1)).astype(F32))
    channel = np.ascontiguousarray(aux[:, k // 16:k // 16 + 4]).view(F32).reshape(n)
    return np.clip(grid, -127, 127).astype(np.int8), channel


def convrot_projection(q, q_scale, grid, channel) -> np.ndarray:
    """``(float(int32 acc) * activation scale) * channel scale`` per output
    (quantized_kernels.py:172-179), fp32; the caller rounds to bf16."""
    acc = q.astype(np.int64) @ grid.astype(np.int64).T
    return ((acc.astype(F32) * np.asarray(q_scale, F32)[:, None]).astype(F32)
            * np.asarray(channel, F32)[None, :]).astype(F32)


def convrot_pairs(x, ids, weights, bank, mode: int, dtype: str = "bfloat16"):
    """``QuantizedExpertBackend(mode)._pairs`` (quantized_kernels.py:230-245) on
    the GPU kernel's semantics: weighted fp32 partials [P, H].

    up = bf16(projection(rotate_quantize(x), W13)); act = bf16(bf16(silu(gate)) * up);
    down = bf16(projection(rotate_quantize(act), W2)) * weight.
    """
    x = np.asarray(x, dtype=F32)
    ids = np.asarray(ids, dtype=np.int64).reshape(-1)
    weights = np.asarray(weights, dtype=F32).reshape(-1)
    hidden = x.shape[1]
    inter = bank["w13_weight"].shape[1] // 2
    qx, sx = quantize_rows_int8(convrot_rotate(x, dtype))
    out = np.zeros((ids.size, hidden), dtype=F32)
    grids: dict[int, tuple] = {}
    for row, slot in enumerate(ids.tolist()):
        if slot not in grids:
            grids[slot] = (convrot_grid(bank["w13_weight"][slot], bank["w13_scale_inv"][slot], mode, hidden),
                           convrot_grid(bank["w2_weight"][slot], bank["w2_scale_inv"][slot], mode, inter))
        (g13, c13), (g2, c2) = grids[slot]
        gu = round_to(convrot_projection(qx[row:row + 1], sx[row:row + 1], g13, c13)[0], dtype)
        act = round_to(round_to(silu(gu[:inter]), dtype) * gu[inter:], dtype)
        qh, sh = quantize_rows_int8(convrot_rotate(act[None, :], dtype))
        down = round_to(convrot_projection(qh, sh, g2, c2)[0], dtype)
        out[row] = (down * weights[row]).astype(F32)
    return out


def convrot_forward(x, ids, weights, bank, mode: int, dtype: str = "bfloat16"):
    """``QuantizedExpertBackend(mode).forward`` (quantized_kernels.py:222-229):
    per-token rows repeated over the route slots, partials summed in slot order."""
    x = np.asarray(x, dtype=F32)
    tokens, top_k = np.asarray(ids).shape
    pairs = convrot_pairs(np.repeat(x, top_k, axis=0), np.asarray(ids).reshape(-1),
                       np.asarray(weights).reshape(-1), bank, mode, dtype)
    return combine_slots(pairs, tokens, top_k, dtype)


# --------------------------------------------------------------------------
# Shared expert + gate and the post-MoE sum (backbone_graph.py:327-337)
# --------------------------------------------------------------------------


def shared_expert(x, gate_proj, up_proj, down_proj, gate_weight):
    """``sigmoid(shared_expert_gate(x)) * shared_expert(x)`` with bf16 modules:
    each Linear rounds to bf16, silu and the products round to bf16."""
    x = np.asarray(x, dtype=F32)
    gate = round_bf16(x @ np.asarray(gate_proj, F32).T)
    up = round_bf16(x @ np.asarray(up_proj, F32).T)
    h = round_bf16(round_bf16(silu(gate)) * up)
    d = round_bf16(h @ np.asarray(down_proj, F32).T)
    logit = round_bf16(x @ np.asarray(gate_weight, F32).reshape(-1, 1))
    with np.errstate(over="ignore"):
        s = round_bf16((F32(1.0) / (F32(1.0) + np.exp(-logit).astype(F32))).astype(F32))
    return round_bf16(s * d)


def post_moe(after_mixer, expert_output, shared):
    """``after_mixer + (expert_output + shared)`` in bf16 (``_post_impl``)."""
    t = round_bf16(np.asarray(expert_output, F32) + np.asarray(shared, F32))
    return round_bf16(np.asarray(after_mixer, F32) + t)
