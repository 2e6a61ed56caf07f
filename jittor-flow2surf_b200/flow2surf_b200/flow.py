"""Integration schedule of the reverse flow (flow2surf/flow.py:24-52), host-side NumPy."""

import numpy as np


def alpha_schedule(num_steps, clean_power, noisy_power):
    """Endpoint-controlled integration levels (flow.py:24-52):
    alpha_i = s_i^clean / (s_i^clean + (1 - s_i)^noisy), s_i = i / num_steps,
    float32, strictly increasing."""
    num_steps = int(num_steps)
    if num_steps < 1:
        raise ValueError("num_steps must be >= 1")
    clean_power = float(clean_power)
    noisy_power = float(noisy_power)
    for name, value in (("clean_power", clean_power), ("noisy_power", noisy_power)):
        if not np.isfinite(value) or value <= 0:
            raise ValueError(f"{name} must be finite and positive, got {value}")
    s = np.arange(1, num_steps + 1, dtype=np.float64) / num_steps
    clean_term = s**clean_power
    noisy_term = (1.0 - s) ** noisy_power
    alpha = (clean_term / (clean_term + noisy_term)).astype(np.float32)
    if not np.isfinite(alpha).all() or alpha[0] <= 0 or np.any(np.diff(alpha) <= 0):
        raise ValueError("schedule parameters must produce strictly increasing positive "
                         "float32 levels")
    return alpha
