"""Property test (hypothesis) of the oracle's per-tensor update in its torch-CPU form against
the reference's op sequence run by torch on CPU (oracle/torch_ops.py, bit for bit the
reference on the golden cases), over random dtypes, sizes, learning rates, weight decays,
step counts, betas, eps, clip factors and value scales -- beyond the golden cases' settings.
exp_avg and exp_avg_sq bit for bit; master within 2 ulp or 1e-6 of its RMS (torch's CPU sqrt
is MKL's, within 1 ulp of correctly rounded); the low-precision copy is RNE of the master."""
import numpy as np
from hypothesis import example, given, settings
from hypothesis import strategies as st

from helpers import assert_bits_equal, assert_state_close, to_numpy, to_torch
from oracle import zero1 as Z
from oracle.torch_ops import adamw_tensor_

log_uniform = lambda lo, hi: st.floats(min_value=np.log10(lo), max_value=np.log10(hi)).map(lambda e: 10.0 ** e)


@settings(max_examples=200, deadline=None)
@given(dtype=st.sampled_from([Z.F32, Z.BF16, Z.F16]), n=st.integers(min_value=1, max_value=3000),
       lr=log_uniform(1e-7, 1e-2), wd=st.one_of(st.just(0.0), st.floats(min_value=0.0, max_value=0.2)),
       step=st.integers(min_value=1, max_value=20000), beta1=st.floats(min_value=0.8, max_value=0.95),
       beta2=st.floats(min_value=0.95, max_value=0.9999), eps=st.sampled_from([1e-8, 1e-6]),
       clip=st.one_of(st.none(), st.floats(min_value=0.01, max_value=1.0)), gsig=log_uniform(1e-6, 1.0),
       seed=st.integers(min_value=0, max_value=2**31))
# an update term 3.7x lr taking the master to ~6e-4: the two sqrt roundings differ by an ulp of
# the term, 64 ulps of the master
@example(dtype=Z.F32, n=1591, lr=0.01, wd=0.0, step=505, beta1=0.8125, beta2=0.9662377480956827, eps=1e-8,
         clip=0.9196285892387314, gsig=0.01, seed=116)
def test_oracle_cpu_form_matches_torch_cpu(dtype, n, lr, wd, step, beta1, beta2, eps, clip, gsig, seed):
    import torch
    rng = np.random.default_rng(seed)
    g32 = (rng.standard_normal(n) * gsig).astype(np.float32)
    master = (rng.standard_normal(n) * 0.02).astype(np.float32)
    m = (rng.standard_normal(n) * gsig * 0.1).astype(np.float32)
    v = np.abs(rng.standard_normal(n) * gsig * gsig * 0.1).astype(np.float32)
    g = Z.narrow(g32, dtype, Z.FORM_TORCH_CPU)
    param = None if dtype == Z.F32 else Z.narrow(master, dtype, Z.FORM_TORCH_CPU)
    # the oracle
    om, oea, oeas = master.copy(), m.copy(), v.copy()
    op = None if param is None else param.copy()
    Z.adamw_tensor(Z.FORM_TORCH_CPU, g, dtype, om, oea, oeas, op, dtype, lr=lr, beta1=beta1, beta2=beta2, eps=eps,
                   weight_decay=wd, step=step, clip_scale=clip)
    # the reference's ops on CPU: the in-place clip, then the update
    tg = to_torch(g, dtype)
    if clip is not None:
        tg.mul_(clip)
    tmaster = torch.from_numpy(master.copy())
    tm, tv = torch.from_numpy(m.copy()), torch.from_numpy(v.copy())
    tparam = tmaster if param is None else to_torch(param, dtype)
    adamw_tensor_(tparam, tg, tmaster, tm, tv, lr=lr, betas=(beta1, beta2), eps=eps, weight_decay=wd, step=step,
                  master_is_parameter=param is None)
    assert_bits_equal(oea, tm.numpy(), "exp_avg")
    assert_bits_equal(oeas, tv.numpy(), "exp_avg_sq")
    # the oracle's correctly rounded sqrt vs MKL's on this host: the update term may move by an
    # ulp of itself (the documented master exception), visible only where the master is near zero
    m_hat = oea.astype(np.float64) / (1 - beta1 ** step)
    v_hat = oeas.astype(np.float64) / (1 - beta2 ** step)
    term = np.maximum(lr * np.abs(m_hat) / (np.sqrt(v_hat) + eps), lr)
    assert_state_close(om, tmaster.numpy(), "master", lr_ulps=(term, 2))
    if param is not None:
        assert_bits_equal(op, Z.narrow(om, dtype, Z.FORM_TORCH_CPU), "param = RNE(master)")
        assert_bits_equal(to_numpy(tparam, dtype), Z.narrow(tmaster.numpy(), dtype, Z.FORM_TORCH_CPU),
                          "reference param = RNE(master)")
