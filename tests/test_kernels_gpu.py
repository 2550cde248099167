"""Parity of each CUDA kernel, called through the C ABI, against the CPU oracle.

AdamW and the in-place clip: bit for bit against the oracle's torch-CUDA form (which
tests/test_torch_cuda_forms.py pins to torch's own CUDA kernels).  Sum of squares:
within 1e-7 relative of the exact fp64 sum, bit-identical across repeated launches.
Edge cases: every tail length, 1-element tensors, tensors larger than one chunk,
unaligned caller pointers (scalar path), entries without a gradient, per-tensor lr and
step, empty launches, NaN / Inf propagation.
"""
import ctypes

import numpy as np
import pytest

from helpers import BF16, F16, F32, Z, assert_bits_equal, to_numpy, to_torch
from hybridagent_b200 import _lib, layout

pytestmark = pytest.mark.gpu

SIZES = [1, 3, 4, 5, 7, 8, 9, 63, 64, 65, 1000, 4095, 4096, 4097, 16383, 16384, 16385, 50001, 65536, 100003]
B1, B2, EPS = 0.9, 0.999, 1e-8


def _dev_bytes(a: np.ndarray):
    import torch
    return torch.from_numpy(a.view(np.uint8).copy()).cuda()


class Tensors:
    """Device buffers + ha_tensor table for a list of tensors of one dtype."""

    def __init__(self, code, sizes, seed, *, misalign=(), no_grad=(), grad_sigma=1e-2, lr=None, steps=None):
        import torch
        rng = np.random.default_rng(seed)
        self.code, self.sizes = code, sizes
        self.keep = []
        n = len(sizes)
        self.lrs = np.array(lr if lr is not None else [1e-3 * (1 + k % 3) for k in range(n)], np.float64)
        self.steps = np.array(steps if steps is not None else [1 + 37 * k for k in range(n)], np.int64)
        self.np_grad, self.np_master, self.np_m, self.np_v, self.np_param = [], [], [], [], []
        self.grad, self.master, self.m, self.v, self.param = [], [], [], [], []
        for k, size in enumerate(sizes):
            master = (rng.standard_normal(size) * 0.02).astype(np.float32)
            m = (rng.standard_normal(size) * 1e-3).astype(np.float32)
            v = np.abs(rng.standard_normal(size) * 1e-5).astype(np.float32)
            g = Z.narrow((rng.standard_normal(size) * grad_sigma).astype(np.float32), code)
            param = None if code == F32 else Z.narrow(master, code)
            self.np_grad.append(None if k in no_grad else g)
            self.np_master.append(master)
            self.np_m.append(m)
            self.np_v.append(v)
            self.np_param.append(param)
            if k in no_grad:
                self.grad.append(None)
            else:
                gt = to_torch(g, code, device="cuda")
                if k in misalign:  # view starting one element into a larger buffer
                    big = torch.zeros(size + 1, dtype=gt.dtype, device="cuda")
                    big[1:].copy_(gt)
                    self.keep.append(big)
                    gt = big[1:]
                self.grad.append(gt)
            self.master.append(to_torch(master, F32, device="cuda"))
            self.m.append(to_torch(m, F32, device="cuda"))
            self.v.append(to_torch(v, F32, device="cuda"))
            if code == F32:
                self.param.append(None)
            else:
                pt = to_torch(param, code, device="cuda")
                if k in misalign:
                    big = torch.zeros(size + 1, dtype=pt.dtype, device="cuda")
                    big[1:].copy_(pt)
                    self.keep.append(big)
                    pt = big[1:]
                self.param.append(pt)
        tab = np.zeros(n, dtype=_lib.TENSOR_DTYPE)
        for k in range(n):
            tab[k]["grad"] = 0 if self.grad[k] is None else self.grad[k].data_ptr()
            tab[k]["master"] = self.master[k].data_ptr()
            tab[k]["exp_avg"] = self.m[k].data_ptr()
            tab[k]["exp_avg_sq"] = self.v[k].data_ptr()
            tab[k]["param"] = 0 if self.param[k] is None else self.param[k].data_ptr()
            tab[k]["numel"] = sizes[k]
        self.tab = tab

    def device_table(self, wd):
        _lib.call("ha_fill_step_scalars", len(self.sizes), _lib.np_ptr(self.lrs), _lib.np_ptr(self.steps), B1, B2, wd,
                  _lib.np_ptr(self.tab))
        return _dev_bytes(self.tab)


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def _adamw(ts: Tensors, wd: float, clip_scale):
    import torch
    table = ts.device_table(wd)
    chunks = layout.chunk_table(ts.sizes, _lib.HA_ADAMW_CHUNK)
    dchunks = _dev_bytes(chunks)
    sc = _lib.AdamwScalars()
    _lib.call("ha_make_scalars", B1, B2, EPS, wd, ts.code, clip_scale is not None,
              0.0 if clip_scale is None else clip_scale, ctypes.byref(sc))
    _lib.call("ha_adamw_step", table.data_ptr(), dchunks.data_ptr(), len(chunks), _lib.HA_ADAMW_CHUNK, ts.code, ts.code,
              ctypes.byref(sc), _stream())
    torch.cuda.synchronize()


def _check_adamw(ts: Tensors, wd: float, clip_scale):
    for k in range(len(ts.sizes)):
        master, m, v = ts.np_master[k].copy(), ts.np_m[k].copy(), ts.np_v[k].copy()
        param = None if ts.np_param[k] is None else ts.np_param[k].copy()
        if ts.np_grad[k] is not None:
            Z.adamw_tensor(Z.FORM_TORCH_CUDA, ts.np_grad[k], ts.code, master, m, v, param, ts.code,
                           lr=float(ts.lrs[k]), beta1=B1, beta2=B2, eps=EPS, weight_decay=wd,
                           step=int(ts.steps[k]), clip_scale=clip_scale)
        assert_bits_equal(to_numpy(ts.master[k], F32), master, f"master[{k}] n={ts.sizes[k]}")
        assert_bits_equal(to_numpy(ts.m[k], F32), m, f"exp_avg[{k}] n={ts.sizes[k]}")
        assert_bits_equal(to_numpy(ts.v[k], F32), v, f"exp_avg_sq[{k}] n={ts.sizes[k]}")
        if param is not None:
            assert_bits_equal(to_numpy(ts.param[k], ts.code), param, f"param[{k}] n={ts.sizes[k]}")


@pytest.mark.parametrize("code", [BF16, F16, F32], ids=["bf16", "f16", "f32"])
@pytest.mark.parametrize("clip", [None, 0.3712345], ids=["noclip", "clip"])
@pytest.mark.parametrize("wd", [0.01, 0.0], ids=["wd", "nowd"])
def test_adamw_matches_oracle(code, clip, wd):
    ts = Tensors(code, SIZES, seed=11 + code, misalign=(4, 13), no_grad=(2, 17))
    _adamw(ts, wd, clip)
    _check_adamw(ts, wd, clip)


def test_adamw_large_values_and_nonfinite():
    """Gradients with inf / nan / huge values and a clip factor of 0 (the reference's
    +inf-norm case) propagate exactly like the oracle."""
    ts = Tensors(BF16, [4096, 777], seed=5, grad_sigma=1e3)
    import torch
    g0 = ts.np_grad[0]
    g0[[3, 100, 2000]] = Z.to_bf16(np.array([np.inf, -np.inf, np.nan], np.float32))
    ts.grad[0].copy_(to_torch(g0, BF16, device="cuda"))
    _adamw(ts, 0.01, 0.0)
    _check_adamw(ts, 0.01, 0.0)
    torch.cuda.synchronize()


@pytest.mark.parametrize("code", [BF16, F16, F32], ids=["bf16", "f16", "f32"])
def test_grad_sumsq(code):
    import torch
    ts = Tensors(code, SIZES + [3 * 32768 + 5], seed=3 + code, misalign=(6,), no_grad=(1,))
    table = ts.device_table(0.0)
    chunks = layout.chunk_table(ts.sizes, _lib.HA_SUMSQ_CHUNK)
    dchunks = _dev_bytes(chunks)
    partials = torch.empty(len(chunks), dtype=torch.float64, device="cuda")
    out = torch.empty(1, dtype=torch.float64, device="cuda")
    results = []
    for _ in range(3):
        _lib.call("ha_grad_sumsq", table.data_ptr(), dchunks.data_ptr(), len(chunks), _lib.HA_SUMSQ_CHUNK, code,
                  partials.data_ptr(), out.data_ptr(), _stream())
        results.append(out.item())
    exact = sum(Z.sumsq(g, code) for g in ts.np_grad if g is not None)
    assert results[0] == results[1] == results[2]  # deterministic
    # fp32 pairwise sums of 16-byte vectors, fp64 above: ~1e-8 relative, below the
    # fp32 rounding of the total that the norm is taken from
    assert abs(results[0] - exact) <= 1e-7 * exact


@pytest.mark.parametrize("code", [BF16, F32], ids=["bf16", "f32"])
def test_grad_sumsq_capped_grid_is_bit_identical(code):
    """ha_grad_sumsq_ctas: every CTA cap (1, a few, fewer than the chunks, more than the
    chunks) gives the partials and the sum of the one-CTA-per-chunk launch, bit for bit."""
    import torch
    ts = Tensors(code, SIZES + [5 * 32768 + 3], seed=31 + code, misalign=(6,), no_grad=(1,))
    table = ts.device_table(0.0)
    chunks = layout.chunk_table(ts.sizes, _lib.HA_SUMSQ_CHUNK)
    dchunks = _dev_bytes(chunks)
    n = len(chunks)
    base_p = torch.empty(n, dtype=torch.float64, device="cuda")
    base = torch.empty(1, dtype=torch.float64, device="cuda")
    _lib.call("ha_grad_sumsq", table.data_ptr(), dchunks.data_ptr(), n, _lib.HA_SUMSQ_CHUNK, code,
              base_p.data_ptr(), base.data_ptr(), _stream())
    for cap in (1, 3, 16, max(n - 1, 1), n + 7, 0):
        p = torch.full((n,), float("nan"), dtype=torch.float64, device="cuda")
        out = torch.empty(1, dtype=torch.float64, device="cuda")
        _lib.call("ha_grad_sumsq_ctas", table.data_ptr(), dchunks.data_ptr(), n, _lib.HA_SUMSQ_CHUNK, code,
                  p.data_ptr(), out.data_ptr(), cap, _stream())
        torch.cuda.synchronize()
        assert torch.equal(p.view(torch.int64), base_p.view(torch.int64)), cap
        assert out.item() == base.item(), cap
    with pytest.raises(RuntimeError):
        _lib.call("ha_grad_sumsq_ctas", table.data_ptr(), dchunks.data_ptr(), n, _lib.HA_SUMSQ_CHUNK, code,
                  base_p.data_ptr(), base.data_ptr(), -1, _stream())


def test_grad_sumsq_nonfinite_and_empty():
    import torch
    ts = Tensors(BF16, [1000, 70000], seed=9)
    out = torch.empty(1, dtype=torch.float64, device="cuda")
    partials = torch.empty(8, dtype=torch.float64, device="cuda")
    # empty launch writes 0
    _lib.call("ha_grad_sumsq", None, None, 0, _lib.HA_SUMSQ_CHUNK, BF16, partials.data_ptr(), out.data_ptr(), _stream())
    assert out.item() == 0.0
    table = ts.device_table(0.0)
    chunks = _dev_bytes(layout.chunk_table(ts.sizes, _lib.HA_SUMSQ_CHUNK))
    n = len(layout.chunk_table(ts.sizes, _lib.HA_SUMSQ_CHUNK))
    for bad, check in ((np.inf, np.isposinf), (np.nan, np.isnan)):
        g = ts.np_grad[1].copy()
        g[12345] = Z.to_bf16(np.array([bad], np.float32))[0]
        ts.grad[1].copy_(to_torch(g, BF16, device="cuda"))
        _lib.call("ha_grad_sumsq", table.data_ptr(), chunks.data_ptr(), n, _lib.HA_SUMSQ_CHUNK, BF16,
                  partials.data_ptr(), out.data_ptr(), _stream())
        assert check(out.item())


@pytest.mark.parametrize("code", [BF16, F32], ids=["bf16", "f32"])
def test_scale_grads(code):
    import torch
    ts = Tensors(code, SIZES, seed=21, misalign=(3,), no_grad=(5,))
    table = ts.device_table(0.0)
    chunks = layout.chunk_table(ts.sizes, _lib.HA_ADAMW_CHUNK)
    scale = 1.0 / (2.7182818 + 1e-6)
    mult = Z.clip_multiplier(code, Z.FORM_TORCH_CUDA, scale)
    dchunks = _dev_bytes(chunks)
    _lib.call("ha_scale_grads", table.data_ptr(), dchunks.data_ptr(), len(chunks), _lib.HA_ADAMW_CHUNK, code, mult,
              _stream())
    torch.cuda.synchronize()
    for k, g in enumerate(ts.np_grad):
        if g is None:
            continue
        want = g.copy()
        Z.clip_inplace(want, code, Z.FORM_TORCH_CUDA, scale)
        assert_bits_equal(to_numpy(ts.grad[k], code), want, f"grad[{k}]")


@pytest.mark.parametrize("how", ["per_chunk", "capped1", "capped3", "capped64", "copy_engine"])
@pytest.mark.parametrize("elem", [2, 4])
def test_gather(elem, how):
    """ha_gather (one CTA per chunk), ha_gather_capped (a grid of 1, 3 or 64 CTAs walking the
    chunk list) and ha_copy_async (copy engines) make the same copies and zero-fills."""
    import torch
    dt = torch.bfloat16 if elem == 2 else torch.float32
    sizes = [5, 16384, 16385, 40000, 1, 0, 333]
    srcs = [torch.randn(n, device="cuda").to(dt) for n in sizes]
    dst = torch.full((sum(sizes) + 64 * len(sizes),), 7.0, device="cuda").to(dt)
    offs, o = [], 0
    for n in sizes:
        offs.append(o)
        o += n + (3 if len(offs) % 2 else 64)  # some destinations unaligned
    tab = np.zeros(len(sizes), dtype=_lib.COPY_DTYPE)
    for k, (n, s) in enumerate(zip(sizes, srcs)):
        tab[k]["src"] = 0 if k == 3 else s.data_ptr()  # entry 3: zero fill
        tab[k]["dst"] = dst.data_ptr() + offs[k] * elem
        tab[k]["numel"] = n
    chunks = layout.chunk_table(sizes, 16384)
    dtab, dchunks = _dev_bytes(tab), _dev_bytes(chunks)  # device tables must outlive the launch
    if how == "per_chunk":
        _lib.call("ha_gather", dtab.data_ptr(), dchunks.data_ptr(), len(chunks), 16384, elem, _stream())
    elif how == "copy_engine":
        _lib.call("ha_copy_async", _lib.np_ptr(tab), len(tab), elem, _stream())
    else:
        _lib.call("ha_gather_capped", dtab.data_ptr(), dchunks.data_ptr(), len(chunks), 16384, elem,
                  int(how[len("capped"):]), _stream())
    torch.cuda.synchronize()
    for k, n in enumerate(sizes):
        got = dst[offs[k]:offs[k] + n]
        want = torch.zeros_like(got) if k == 3 else srcs[k]
        assert torch.equal(got.view(torch.int16 if elem == 2 else torch.int32),
                           want.view(torch.int16 if elem == 2 else torch.int32)), k


@pytest.mark.parametrize("entry", ["delta_peers", "delta_local", "dense_peers"])
@pytest.mark.parametrize("code", [BF16, F16], ids=["bf16", "f16"])
def test_adamw_peer_and_changed_group_stores(code, entry):
    """Parameter stores of the fused update, with two 'peers' emulated on this GPU (arenas at
    fixed offsets from the local parameter arena).  ha_adamw_step_delta: the local parameters
    (and, with peers, every peer) end with the oracle's new values wherever a 4-element group
    (per element on the scalar path and ragged tails) changed its rounded value, the other groups
    of its 32-byte sector with it; groups in unchanged sectors are not stored at all -- a sentinel
    planted in a peer's copy there survives, one in a changed sector is overwritten.
    ha_adamw_step_peers stores every group."""
    import torch
    sizes = SIZES + [3 * 16384 + 6]
    n = len(sizes)
    rng = np.random.default_rng(40 + code)
    # half the tensors with a large learning rate (most rounded values move), half tiny (few do)
    lrs = [1e-3 if k % 2 == 0 else 1e-9 for k in range(n)]
    ts = Tensors(code, sizes, seed=30 + code, misalign=(4, 13), no_grad=(2, 17), lr=lrs)
    offs, o = [], 0
    for k, size in enumerate(sizes):
        o += 1 if k in (4, 13) else 0  # the misaligned tensors keep an odd start in the arena
        offs.append(o)
        o = (o + size + 63) // 64 * 64
    dt = ts.param[0].dtype
    local = torch.zeros(o, dtype=dt, device="cuda")
    for k, size in enumerate(sizes):
        local[offs[k]:offs[k] + size].copy_(ts.param[k])
        ts.tab[k]["param"] = local.data_ptr() + 2 * offs[k]
    init = to_numpy(local, code)
    peers = [torch.zeros(o, dtype=dt, device="cuda") for _ in range(2)]
    planted = rng.choice(o, size=4000, replace=False)
    peer_init = []
    for p in peers:
        bits = init.copy()
        bits[planted] ^= 1  # sentinels: a peer copy that differs from the local one
        p.copy_(to_torch(bits, code, device="cuda"))
        peer_init.append(bits)
    pe = _lib.Peers()
    pe.n = 2
    for q, p in enumerate(peers):
        pe.delta[q] = p.data_ptr() - local.data_ptr()
    table = ts.device_table(0.01)
    chunks = layout.chunk_table(sizes, _lib.HA_ADAMW_CHUNK)
    dchunks = _dev_bytes(chunks)
    sc = _lib.AdamwScalars()
    _lib.call("ha_make_scalars", B1, B2, EPS, 0.01, code, 0, 0.0, ctypes.byref(sc))
    if entry == "dense_peers":
        _lib.call("ha_adamw_step_peers", table.data_ptr(), dchunks.data_ptr(), len(chunks), _lib.HA_ADAMW_CHUNK, code,
                  code, ctypes.byref(sc), ctypes.byref(pe), _stream())
    else:
        cnt = torch.zeros(1, dtype=torch.int64, device="cuda")
        _lib.call("ha_adamw_step_delta", table.data_ptr(), dchunks.data_ptr(), len(chunks), _lib.HA_ADAMW_CHUNK, code,
                  ctypes.byref(sc), ctypes.byref(pe) if entry == "delta_peers" else None, cnt.data_ptr(), _stream())
    torch.cuda.synchronize()
    want_count = 0
    got_local = to_numpy(local, code)
    got_peers = [to_numpy(p, code) for p in peers]
    changed_any = 0
    for k, size in enumerate(sizes):
        master, m, v = ts.np_master[k].copy(), ts.np_m[k].copy(), ts.np_v[k].copy()
        param = ts.np_param[k].copy()
        if ts.np_grad[k] is not None:
            Z.adamw_tensor(Z.FORM_TORCH_CUDA, ts.np_grad[k], code, master, m, v, param, code, lr=float(ts.lrs[k]),
                           beta1=B1, beta2=B2, eps=EPS, weight_decay=0.01, step=int(ts.steps[k]), clip_scale=None)
        sl = slice(offs[k], offs[k] + size)
        old = init[sl]
        assert_bits_equal(got_local[sl], param, f"local param[{k}]")
        # which elements were stored: the element's 4-group changed (vector path: whole groups of
        # an aligned tensor), or the element itself (scalar path, ragged tail)
        diff = param != old
        stored = diff.copy()
        if entry == "dense_peers":
            stored[:] = ts.np_grad[k] is not None
        elif ts.np_grad[k] is not None and k not in (4, 13):
            # vector path: 4-element groups; the four groups of a 32-byte sector (16 elements) are
            # stored together when any of them changed
            full = size // 4 * 4
            grp = diff[:full].reshape(-1, 4).any(axis=1)
            quad = np.zeros(-(-len(grp) // 4) * 4, dtype=bool)
            quad[:len(grp)] = grp
            quad = np.repeat(quad.reshape(-1, 4).any(axis=1), 4)[:len(grp)]
            stored[:full] = np.repeat(quad, 4)
            want_count += int(quad.sum()) + int(diff[full:].sum())
        elif ts.np_grad[k] is not None:
            want_count += int(diff.sum())  # scalar path: one per changed element
        if entry == "delta_local":
            stored[:] = False  # no peer is written
        changed_any += int(diff.sum())
        for q in range(2):
            want = np.where(stored, param, peer_init[q][sl])
            assert_bits_equal(got_peers[q][sl], want, f"peer {q} param[{k}]")
    assert changed_any > 1000  # the large-lr tensors moved
    if entry != "dense_peers":
        assert int(cnt.item()) == want_count  # the groups the kernel counts as stored
        survived = int((got_peers[0][planted] == peer_init[0][planted]).sum())
        assert survived > 1000  # most sentinels sat in unchanged groups of the tiny-lr tensors
