"""Shared helpers for the parity tests (CUDA path vs CPU oracle)."""

import numpy as np

OUT_MAX_ABS = 2e-3      # attention output max-abs
OUT_MIN_COS = 0.9999    # and cosine
TIE_EPS = 1e-3          # score gap below which a spike decision is a numerical tie


def np_(t):
    return t.detach().cpu().numpy()


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint16) if a.dtype == np.float16 else a


def layer_to_oracle(lay, tc=None):
    """FoveatedLayer (torch) -> the dict layout fkv_oracle.decode_attend expects."""
    d = {"near_k": np_(lay.near_k), "near_v": np_(lay.near_v),
         "near_valid": np_(lay.near_valid), "compress_method": lay.compress_method,
         "v_group": lay.v_group}
    if lay.compress_method == "turbo":
        d.update(turbo_k_idx=np_(lay.turbo_far_k_indices), turbo_k_signs=np_(lay.turbo_far_k_signs),
                 turbo_k_norm=np_(lay.turbo_far_k_norm), turbo_k_gamma=np_(lay.turbo_far_k_gamma),
                 turbo_v_packed=np_(lay.turbo_far_v_packed), turbo_v_scale=np_(lay.turbo_far_v_scale),
                 tc=tc)
    else:
        d.update(far_k=np_(lay.far_k), far_v=np_(lay.far_v), far_v_scale=np_(lay.far_v_scale),
                 far_v_zero=np_(lay.far_v_zero))
    return d


def assert_output_close(out, ref, what=""):
    out = np.asarray(out, dtype=np.float64).reshape(ref.shape)
    err = np.abs(out - ref).max()
    cos = (out * ref).sum() / np.sqrt((out * out).sum() * (ref * ref).sum() + 1e-300)
    assert err <= OUT_MAX_ABS, f"{what}: max-abs {err:.3e} > {OUT_MAX_ABS}"
    assert cos >= OUT_MIN_COS, f"{what}: cosine {cos:.6f} < {OUT_MIN_COS}"
    return err, cos


def assert_spikes_match(flags, tokens, rflags, rtokens, diag, margin, what=""):
    """Flags and tokens must be identical except where the oracle's own scores
    sit within TIE_EPS of the decision (flag) or of the runner-up (token).
    Returns the number of such tie cases (expected 0 on seeded data)."""
    flags = np.asarray(flags).reshape(rflags.shape)
    tokens = np.asarray(tokens).reshape(rtokens.shape)
    ties = 0
    bad_f = np.argwhere(flags != rflags)
    for idx in bad_f:
        gap = abs(diag["max_far"][tuple(idx)] - (diag["min_near"][tuple(idx)] + margin))
        assert gap < TIE_EPS, f"{what}: flag mismatch at {tuple(idx)} (gap {gap})"
        ties += 1
    bad_t = np.argwhere(tokens != rtokens)
    for idx in bad_t:
        gap = abs(diag["max_far"][tuple(idx)] - diag["second_far"][tuple(idx)])
        assert gap < TIE_EPS, f"{what}: token mismatch at {tuple(idx)} (gap {gap})"
        ties += 1
    return ties
