"""Shape constants of the Qwen3-8B attention block and the parity
tolerances, shared by the tests."""
HQ, HKV, HD = 32, 8, 128
KV_DIM = HKV * HD
KV_MUL = HQ // HKV
EPS, THETA = 1e-6, 5e6

# fp32 cache: normwise max relative error ||gpu - ref||_inf / ||ref||_inf
TOL_F32_NORMWISE = 2e-4
# bf16 cache: max absolute error against the reference fed the same
# bf16-rounded K/V
TOL_BF16_ABS = 1e-2


def normwise(a, b):
    import numpy as np
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def elementwise_floor(a, b, tau_frac=1e-3):
    """max |a-b| / max(|b|, tau) with tau = tau_frac * ||b||_inf."""
    import numpy as np
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    tau = tau_frac * np.abs(b).max()
    return float((np.abs(a - b) / np.maximum(np.abs(b), tau)).max())
