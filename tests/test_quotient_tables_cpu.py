"""CPU checks of the arithmetic facts the GPU quantizers' quotient tables rely
on (no GPU needed).

* The vision-aware quantizer's output x + (q/s - x) (quant_rpfq_vit_vision.py:
  156-167) does not depend on the sign of a zero quotient, so its table may
  hold one zero entry for q = +0 and q = -0.
* ActivationQuantSTE's output is q/s itself (quant_i.py:442-455), and rint of a
  small negative value is -0, so its table needs a separate -0 slot."""

import numpy as np


def test_vision_output_ignores_sign_of_zero_quotient():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(4096).astype(np.float32) * 1e-3,
                        np.array([0.0, -0.0, 1e-30, -1e-30, 5e-4, -5e-4], dtype=np.float32)])
    s = np.float32(127.0) / np.float32(2.0)
    q = np.clip(np.rint(x * s), -128, 127).astype(np.float32)
    zero = q == 0
    assert zero.any() and np.signbit(q[zero]).any() and (~np.signbit(q[zero])).any()
    for qx0 in (np.float32(0.0), np.float32(-0.0)):
        qx = np.where(zero, qx0, q / s).astype(np.float32)
        y = (x + (qx - x)).astype(np.float16)
        if qx0 == 0 and not np.signbit(qx0):
            ref = y
        else:
            assert np.array_equal(y.view(np.uint16), ref.view(np.uint16))


def test_act_quant_needs_negative_zero_slot():
    s = np.float32(7.0)  # 4-bit: qmax / amax with amax = 1
    x = np.float32(-0.01)
    q = np.float32(np.clip(np.rint(x * s), -8, 7))
    assert q == 0 and np.signbit(q)
    out = np.float16(q / s)
    assert np.signbit(out)  # -0: a table holding only +0 for q = 0 would flip this bit
