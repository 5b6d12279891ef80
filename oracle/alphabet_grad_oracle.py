"""CPU oracle for the ALPHABET backward pass (numpy restatement of the VJP).

TEST INFRASTRUCTURE ONLY, like ``alphabet_oracle``: the ``-m gpu`` tests use
it to check ``lnet_b200_alphabet_backward``; the product never imports it.

Scope: the eager ``Alphabet.forward`` (src/lnet/alphabet.py:350-416) with
every metadata combination (``time_delta``: physical-time convs and moments;
``observation_mask``, channel or event form; ``valid_mask``); gradients of ``L = sum(logits * dlogits)`` with respect to
every parameter, each frame's gradient taken at the materialised [D, 2M]
weight.  It is pinned against gradients that the reference's own autograd
produces (``tests/golden/make_grad_golden.py``,
``tests/test_grad_oracle.py``).

The VJP of each forward stage, in the order the backward runs:

* head ``logits = feats G^T + b`` (src/lnet/alphabet.py:62-63);
* radial-log features (src/lnet/alphabet.py:29-46): ``R0 = log1p(max(E, 0))``,
  lag pairs ``(re, im) log1p(r) / r`` with ``r = sqrt(max(re^2 + im^2, tiny))``;
* moments (src/lnet/pac_tight_frame_models.py:1632-1702) -> a per-step state
  gradient dS_t (energy term, and each lag pair as the current and as the
  earlier state);
* recurrence ``s_t = a s_{t-1} + u_t`` (src/lnet/pac_recurrence.py:191-212):
  the adjoint runs backwards, ``lambda_t = dS_t + conj(a) lambda_{t+1}``;
  ``du = lambda``; ``da = sum lambda_t conj(s_{t-1})``-type real-pair sums;
* gain ``u = g e`` and the ZOH pole map ``a = exp(p)``, ``g = (a - 1) / p``,
  ``p = -damping + i frequency`` (src/lnet/pac_real2d_math.py:20-53,
  src/lnet/pac_tight_frame_models.py:458-491), by the Cauchy-Riemann form of
  the complex derivatives;
* drive ``e = xhat F`` and, in the writer, synthesis + residual
  ``v = x + ls (s F^T + ds xhat)`` (src/lnet/pac_tight_frame_models.py:1038,
  1480-1507);
* RMSNorm (eps = fp32 eps), depthwise conv K5 d4 + SiLU, masks, the stem
  projection (src/lnet/pac_laplace_native_input.py:98-138,
  src/lnet/alphabet_backbone.py:593-676, 872-992).
"""

from __future__ import annotations

import numpy as np

from .alphabet_oracle import (
    DAMPING_MAX,
    DAMPING_MIN,
    FP32_EPS,
    FP32_TINY,
    LAGS,
    discrete_pole_real2d,
    masked_modal_moments,
    modal_moments,
    physical_time_modal_moments,
    radial_log_lag124,
    recurrence,
    same_length_dwconv,
    searchsorted_left,
    sigmoid,
    timestamps_of,
)


def _conv_taps(x, weight, dilation=4):
    """Zero-padded shifted copies x[t + k dil - pad] for each tap k: [K, B, T, D]."""
    b, t, d = x.shape
    k = weight.shape[-1]
    pad = dilation * (k - 1) // 2
    xp = np.zeros((b, t + 2 * pad, d), dtype=x.dtype)
    xp[:, pad : pad + t] = x
    return np.stack([xp[:, j * dilation : j * dilation + t] for j in range(k)])


def conv_backward(x, weight, dout, dilation=4):
    """VJP of ``same_length_dwconv``: (dx, dweight [D, 1, K], dbias [D])."""
    b, t, d = x.shape
    k = weight.shape[-1]
    pad = dilation * (k - 1) // 2
    w = weight.reshape(d, k)
    taps = _conv_taps(x, weight, dilation)
    dw = np.einsum("btd,kbtd->dk", dout, taps).reshape(d, 1, k)
    db = dout.sum(axis=(0, 1))
    dxp = np.zeros((b, t + 2 * pad, d), dtype=x.dtype)
    for j in range(k):
        dxp[:, j * dilation : j * dilation + t] += dout * w[:, j]
    return dxp[:, pad : pad + t], dw, db


def _lerp_positions(ts, queries):
    """Lower / upper sample index and weight of piecewise-linear lookups at
    ``queries`` (the index arithmetic of _physical_time_depthwise_conv and
    _interpolate_modal_state): [B, Q] each."""
    b, t = ts.shape
    up_u = searchsorted_left(ts, queries)
    upper = np.minimum(up_u, t - 1)
    lower = np.clip(up_u - 1, 0, t - 1)
    bi = np.arange(b)[:, None]
    lt, ut = ts[bi, lower], ts[bi, upper]
    span = ut - lt
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        w = np.where(span > 0, (queries - lt) / np.maximum(span, FP32_TINY), 0.0)
    w = np.clip(w, 0.0, 1.0)
    in_bounds = (queries >= ts[:, :1]) & (queries <= ts[:, -1:])
    return lower, upper, w, in_bounds


def _support(valid, lower, upper, w):
    v = valid[..., 0]
    bi = np.arange(v.shape[0])[:, None]
    lv, uv = v[bi, lower], v[bi, upper]
    eps8 = 8.0 * FP32_EPS
    return np.where(w <= eps8, lv, np.where(w >= 1.0 - eps8, uv, lv * uv))


def physical_conv_parts(x, weight, time_delta, valid, dilation=4):
    """Sample positions of ``physical_time_depthwise_conv``: lower, upper, weight
    and the on-mask per (row, step, tap), each [B, T, K]."""
    b, t, d = x.shape
    k = weight.shape[-1]
    ts = timestamps_of(time_delta[..., 0])
    left = dilation * (k - 1) // 2
    offsets = (np.arange(k) * dilation - left).astype(x.dtype)
    queries = (ts[:, :, None] + offsets[None, None, :]).reshape(b, -1)
    lower, upper, w, on = _lerp_positions(ts, queries)
    if valid is not None:
        on = on & (_support(valid, lower, upper, w) > 0)
    shape = (b, t, k)
    return lower.reshape(shape), upper.reshape(shape), w.reshape(shape), on.reshape(shape)


def physical_conv_forward(x, weight, bias, parts):
    lower, upper, w, on = parts
    b, t, d = x.shape
    bi = np.arange(b)[:, None, None]
    samp = (x[bi, lower] * (1.0 - w)[..., None] + x[bi, upper] * w[..., None]) * on[..., None]
    wk = weight.reshape(d, -1)
    return np.einsum("btkd,dk->btd", samp, wk) + bias.reshape(1, 1, d), samp


def physical_conv_backward(x, weight, parts, samp, dout):
    """VJP of the physical-time conv: dx (scattered onto the lower and upper
    samples with weights 1 - w and w), dweight [D, 1, K], dbias [D]."""
    lower, upper, w, on = parts
    b, t, d = x.shape
    k = weight.shape[-1]
    wk = weight.reshape(d, k)
    dw = np.einsum("btd,btkd->dk", dout, samp).reshape(d, 1, k)
    db = dout.sum(axis=(0, 1))
    dx = np.zeros_like(x)
    for j in range(k):
        g = dout * wk[:, j] * on[..., j, None]
        for bb in range(b):
            np.add.at(dx[bb], lower[bb, :, j], g[bb] * (1.0 - w[bb, :, j, None]))
            np.add.at(dx[bb], upper[bb, :, j], g[bb] * w[bb, :, j, None])
    return dx, dw, db


def physical_moments_backward(s_re, s_im, dm, time_delta, valid):
    """State gradient of ``physical_time_modal_moments`` (duration-weighted
    energy; lag pairs against the state interpolated at t - lag, scattered
    onto its lower and upper samples)."""
    b, t, m = s_re.shape
    delta = time_delta.astype(s_re.dtype)
    valid = np.ones_like(delta) if valid is None else valid.astype(s_re.dtype)
    ts = timestamps_of(delta[..., 0])
    dw_ = delta * valid
    dcount = dw_.sum(axis=1)
    ecount = valid.sum(axis=1)
    use_d = dcount > 0
    ew = np.where(use_d[:, None, :], dw_, valid)
    ec = np.maximum(np.where(use_d, dcount, ecount), 1.0)
    gr = 2.0 * s_re * ew * dm[:, None, :m] / ec[:, None, :]
    gi = 2.0 * s_im * ew * dm[:, None, :m] / ec[:, None, :]
    bi = np.arange(b)[:, None]
    for li, lag in enumerate(LAGS):
        q = (ts - float(lag)).astype(s_re.dtype)
        lower, upper, w, on = _lerp_positions(ts, q)
        sup = _support(valid, lower, upper, w) * on
        pw = (delta[..., 0] * valid[..., 0] * sup)[..., None]
        pc = np.maximum(pw.sum(axis=1, keepdims=True), 1.0)
        dr = dm[:, None, (1 + 2 * li) * m : (2 + 2 * li) * m]
        di = dm[:, None, (2 + 2 * li) * m : (3 + 2 * li) * m]
        wl = w[..., None]
        pr = s_re[bi, lower] * (1.0 - wl) + s_re[bi, upper] * wl
        pi = s_im[bi, lower] * (1.0 - wl) + s_im[bi, upper] * wl
        gr += (dr * pr - di * pi) * pw / pc
        gi += (dr * pi + di * pr) * pw / pc
        hr = (dr * s_re + di * s_im) * pw / pc  # gradient of the interpolated state
        hi = (dr * s_im - di * s_re) * pw / pc
        for bb in range(b):
            np.add.at(gr[bb], lower[bb], hr[bb] * (1.0 - wl[bb]))
            np.add.at(gr[bb], upper[bb], hr[bb] * wl[bb])
            np.add.at(gi[bb], lower[bb], hi[bb] * (1.0 - wl[bb]))
            np.add.at(gi[bb], upper[bb], hi[bb] * wl[bb])
    return gr, gi


def silu_grad(z):
    s = sigmoid(z)
    return s * (1.0 + z * (1.0 - s))


def rms_norm_parts(x, weight):
    rs = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + FP32_EPS)
    return x * rs * weight, rs


def rms_norm_backward(x, rs, weight, dxhat):
    d = x.shape[-1]
    gd = dxhat * weight
    dx = rs * gd - x * rs**3 * np.sum(gd * x, axis=-1, keepdims=True) / d
    dweight = np.sum(dxhat * x * rs, axis=(0, 1))
    return dx, dweight


def radial_log_backward(moments, dfeat, modes):
    """VJP of ``radial_log_lag124``."""
    dm = np.zeros_like(moments)
    e = moments[..., :modes]
    dm[..., :modes] = np.where(e > 0.0, dfeat[..., :modes] / (1.0 + np.maximum(e, 0.0)), 0.0)
    for off in (modes, 3 * modes, 5 * modes):
        re = moments[..., off : off + modes]
        im = moments[..., off + modes : off + 2 * modes]
        gre = dfeat[..., off : off + modes]
        gim = dfeat[..., off + modes : off + 2 * modes]
        q = re * re + im * im
        r = np.sqrt(np.maximum(q, FP32_TINY))
        sc = np.log1p(r) / r
        live = q > FP32_TINY
        kk = np.where(live, (r / (1.0 + r) - np.log1p(r)) / (r * r) / r, 0.0)
        dm[..., off : off + modes] = gre * (sc + re * re * kk) + gim * (im * re * kk)
        dm[..., off + modes : off + 2 * modes] = gre * (re * im * kk) + gim * (sc + im * im * kk)
    return dm


def moments_backward(s_re, s_im, dm, valid=None):
    """State gradient (dS_re, dS_im) [B, T, M] of (masked) modal moments."""
    b, t, m = s_re.shape
    w = np.ones((b, t, 1), dtype=s_re.dtype) if valid is None else valid.astype(s_re.dtype)
    cnt = t if valid is None else np.maximum(w.sum(axis=1, keepdims=True), 1.0)
    de = dm[:, None, :m]
    gr = 2.0 * s_re * de * w / cnt
    gi = 2.0 * s_im * de * w / cnt
    for li, lag in enumerate(LAGS):
        if t <= lag:
            continue
        dr = dm[:, None, (1 + 2 * li) * m : (2 + 2 * li) * m]
        di = dm[:, None, (2 + 2 * li) * m : (3 + 2 * li) * m]
        pw = w[:, lag:] * w[:, :-lag]
        c = (t - lag) if valid is None else np.maximum(pw.sum(axis=1, keepdims=True), 1.0)
        cr, ci = s_re[:, lag:], s_im[:, lag:]
        pr, pi = s_re[:, :-lag], s_im[:, :-lag]
        # as the current state (t >= lag)
        gr[:, lag:] += (dr * pr - di * pi) * pw / c
        gi[:, lag:] += (dr * pi + di * pr) * pw / c
        # as the earlier state (t + lag < T)
        gr[:, :-lag] += (dr * cr + di * ci) * pw / c
        gi[:, :-lag] += (dr * ci - di * cr) * pw / c
    return gr, gi


def scan_backward(a_re, a_im, g_re, g_im, s_re, s_im, ds_re, ds_im, event=None, per_step=False):
    """Adjoint of ``s_t = a s_{t-1} + event_t g e_t``: returns de (re, im) [B, T, M]
    and the per-mode real-pair sums da, dg ([M] each, re and im).  dg uses
    u_t / g with u_t = s_t - a s_{t-1} (the masked drive, so no division by
    the mask).  Coefficients may be per mode or per step ([B, T, M]);
    ``per_step`` returns da, dg per step instead of summed."""
    b, t, m = s_re.shape
    a_re = np.broadcast_to(a_re, s_re.shape)  # per step [B, T, M] or per mode
    a_im = np.broadcast_to(a_im, s_re.shape)
    g_re = np.broadcast_to(g_re, s_re.shape)
    g_im = np.broadcast_to(g_im, s_re.shape)
    lr = np.zeros((b, m), dtype=s_re.dtype)
    li = np.zeros((b, m), dtype=s_re.dtype)
    lam_re = np.empty_like(s_re)
    lam_im = np.empty_like(s_im)
    for i in range(t - 1, -1, -1):
        # lambda_i = dS_i + conj(a_{i+1}) lambda_{i+1}
        nxr = a_re[:, i + 1] if i + 1 < t else 0.0
        nxi = a_im[:, i + 1] if i + 1 < t else 0.0
        nr = ds_re[:, i] + nxr * lr + nxi * li
        ni = ds_im[:, i] + nxr * li - nxi * lr
        lr, li = nr, ni
        lam_re[:, i], lam_im[:, i] = lr, li
    prev_re = np.concatenate([np.zeros_like(s_re[:, :1]), s_re[:, :-1]], axis=1)
    prev_im = np.concatenate([np.zeros_like(s_im[:, :1]), s_im[:, :-1]], axis=1)
    da_re = lam_re * prev_re + lam_im * prev_im  # per step
    da_im = -lam_re * prev_im + lam_im * prev_re
    u_re = s_re - (a_re * prev_re - a_im * prev_im)
    u_im = s_im - (a_im * prev_re + a_re * prev_im)
    den = g_re * g_re + g_im * g_im
    e_re = (u_re * g_re + u_im * g_im) / den
    e_im = (u_im * g_re - u_re * g_im) / den
    dg_re = lam_re * e_re + lam_im * e_im
    dg_im = -lam_re * e_im + lam_im * e_re
    if not per_step:
        da_re, da_im = da_re.sum(axis=(0, 1)), da_im.sum(axis=(0, 1))
        dg_re, dg_im = dg_re.sum(axis=(0, 1)), dg_im.sum(axis=(0, 1))
    de_re = lam_re * g_re + lam_im * g_im
    de_im = -lam_re * g_im + lam_im * g_re
    if event is not None:
        de_re = de_re * event
        de_im = de_im * event
    return de_re, de_im, (da_re, da_im), (dg_re, dg_im)


def pole_backward(raw_decay, raw_frequency, da, dg):
    """d raw_decay, d raw_frequency from the real-pair sums da, dg (dt = 1)."""
    sig = sigmoid(raw_decay)
    damping = DAMPING_MIN + (DAMPING_MAX - DAMPING_MIN) * sig
    th = np.tanh(raw_frequency)
    p = -damping + 1j * (np.pi * th)
    a = np.exp(p)
    fa = a
    fg = (a * p - (a - 1.0)) / (p * p)
    dpr = da[0] * fa.real + da[1] * fa.imag + dg[0] * fg.real + dg[1] * fg.imag
    dpi = -da[0] * fa.imag + da[1] * fa.real - dg[0] * fg.imag + dg[1] * fg.real
    d_raw_decay = -dpr * (DAMPING_MAX - DAMPING_MIN) * sig * (1.0 - sig)
    d_raw_frequency = dpi * np.pi * (1.0 - th * th)
    return d_raw_decay, d_raw_frequency


def pole_backward_steps(raw_decay, raw_frequency, da, dg, dt):
    """d raw_* with per-step da, dg [B, T, M] and steps dt [B, T, 1]:
    a'(p) = dt a, g'(p) = (dt a p - (a - 1)) / p^2 at each step (0 in the
    ZOH's small-|p dt| branch, where g = dt)."""
    sig = sigmoid(raw_decay)
    damping = DAMPING_MIN + (DAMPING_MAX - DAMPING_MIN) * sig
    th = np.tanh(raw_frequency)
    p = -damping + 1j * (np.pi * th)
    a = np.exp(p * dt)
    fa = dt * a
    fg = (dt * a * p - (a - 1.0)) / (p * p)
    fg = np.where(np.abs(p * dt) < 1.0e-6, 0.0, fg)
    dpr = (da[0] * fa.real + da[1] * fa.imag + dg[0] * fg.real + dg[1] * fg.imag).sum(axis=(0, 1))
    dpi = (-da[0] * fa.imag + da[1] * fa.real - dg[0] * fg.imag + dg[1] * fg.real).sum(
        axis=(0, 1))
    d_raw_decay = -dpr * (DAMPING_MAX - DAMPING_MIN) * sig * (1.0 - sig)
    d_raw_frequency = dpi * np.pi * (1.0 - th * th)
    return d_raw_decay, d_raw_frequency


def _block_forward(x, params, prefix, valid, event=None, delta=None):
    g = params[prefix + ".norm.weight"]
    frame = params[prefix + ".frame.weight"]
    m = frame.shape[1] // 2
    xh, rs = rms_norm_parts(x, g)
    e = xh @ frame
    dmp = DAMPING_MIN + (DAMPING_MAX - DAMPING_MIN) * sigmoid(params[prefix + ".raw_decay"])
    frq = np.pi * np.tanh(params[prefix + ".raw_frequency"])
    step = 1.0 if delta is None else delta
    a_re, a_im, g_re, g_im = discrete_pole_real2d(dmp, frq, step, dtype=x.dtype)
    u_re = g_re * e[..., :m] - g_im * e[..., m:]
    u_im = g_re * e[..., m:] + g_im * e[..., :m]
    if event is not None:
        u_re, u_im = event * u_re, event * u_im
    s_re, s_im = recurrence(a_re, a_im, u_re, u_im)
    if delta is not None:
        mom = physical_time_modal_moments(s_re, s_im, delta, valid)
    elif valid is None:
        mom = modal_moments(s_re, s_im)
    else:
        mom = masked_modal_moments(s_re, s_im, valid)
    return dict(xh=xh, rs=rs, a=(a_re, a_im), g=(g_re, g_im), s=(s_re, s_im), mom=mom,
                event=event, delta=delta)


def _block_backward(x, params, prefix, st, dmom, valid, extra_ds=None):
    frame = params[prefix + ".frame.weight"]
    m = frame.shape[1] // 2
    s_re, s_im = st["s"]
    delta = st["delta"]
    if delta is None:
        gr, gi = moments_backward(s_re, s_im, dmom, valid)
    else:
        gr, gi = physical_moments_backward(s_re, s_im, dmom, delta, valid)
    if extra_ds is not None:
        gr = gr + extra_ds[..., :m]
        gi = gi + extra_ds[..., m:]
    de_re, de_im, da, dg = scan_backward(*st["a"], *st["g"], s_re, s_im, gr, gi, st["event"],
                                         per_step=delta is not None)
    de = np.concatenate([de_re, de_im], axis=-1)
    dxh = de @ frame.T
    dframe = np.einsum("btd,btj->dj", st["xh"], de)
    if delta is None:
        draw = pole_backward(params[prefix + ".raw_decay"], params[prefix + ".raw_frequency"],
                             da, dg)
    else:
        draw = pole_backward_steps(params[prefix + ".raw_decay"],
                                   params[prefix + ".raw_frequency"], da, dg, delta)
    return dxh, dframe, draw


def alphabet_backward(x, params, dlogits, *, time_delta=None, observation_mask=None,
                      valid_mask=None, dilation=4, dtype=np.float64):
    """Gradients of ``sum(logits * dlogits)``, keyed like ``state_dict``."""
    p = {k: np.asarray(v, dtype=dtype) for k, v in params.items()}
    x = np.asarray(x, dtype=dtype)
    dlogits = np.asarray(dlogits, dtype=dtype)
    valid = None if valid_mask is None else np.asarray(valid_mask, dtype=dtype)[..., None]
    vm = 1.0 if valid is None else valid
    raw_obs = event = None
    if observation_mask is not None:  # src/lnet/alphabet_backbone.py:538-569
        raw_obs = np.asarray(observation_mask, dtype=dtype)
        if raw_obs.ndim == 2:
            raw_obs = raw_obs[..., None]
        event = raw_obs if raw_obs.shape[-1] == 1 else raw_obs.max(axis=-1, keepdims=True)
    delta = None
    if time_delta is not None:
        delta = np.asarray(time_delta, dtype=dtype)
        delta = delta[..., None] if delta.ndim == 2 else delta
    m = p["forward_block.frame.weight"].shape[1] // 2
    # forward with the saved activations
    stem_in = x * vm if raw_obs is None else x * raw_obs * vm
    proj = stem_in @ p["stem.projection.weight"].T
    if delta is None:
        z1 = same_length_dwconv(proj, p["stem.local.weight"], p["stem.local.bias"], dilation)
    else:
        parts1 = physical_conv_parts(proj, p["stem.local.weight"], delta, valid, dilation)
        z1, samp1 = physical_conv_forward(proj, p["stem.local.weight"], p["stem.local.bias"],
                                          parts1)
    y1 = z1 * sigmoid(z1) * vm
    w_st = _block_forward(y1, p, "forward_block", valid, event, delta)
    s1 = np.concatenate(w_st["s"], axis=-1)
    modal = s1 @ p["forward_block.frame.weight"].T
    ls, ds = p["forward_block.layer_scale"], p["forward_block.direct_scale"]
    v = y1 + ls * (modal + ds * w_st["xh"])
    rin = v * vm
    if delta is None:
        z2 = same_length_dwconv(rin, p["second_local.weight"], p["second_local.bias"], dilation)
    else:
        parts2 = physical_conv_parts(rin, p["second_local.weight"], delta, valid, dilation)
        z2, samp2 = physical_conv_forward(rin, p["second_local.weight"], p["second_local.bias"],
                                          parts2)
    y2 = z2 * sigmoid(z2) * vm
    r_st = _block_forward(y2, p, "backward_block", valid, None, delta)
    feats = np.concatenate([radial_log_lag124(w_st["mom"], m),
                            radial_log_lag124(r_st["mom"], m)], axis=-1)
    head_w = p["head.classifier.weight"]
    grads = {"head.classifier.weight": dlogits.T @ feats,
             "head.classifier.bias": dlogits.sum(axis=0)}
    dfeats = dlogits @ head_w
    dm1 = radial_log_backward(w_st["mom"], dfeats[:, : 7 * m], m)
    dm2 = radial_log_backward(r_st["mom"], dfeats[:, 7 * m :], m)
    # reader
    dxh2, grads["backward_block.frame.weight"], (grads["backward_block.raw_decay"],
                                                 grads["backward_block.raw_frequency"]) = \
        _block_backward(y2, p, "backward_block", r_st, dm2, valid)
    dy2, grads["backward_block.norm.weight"] = rms_norm_backward(
        y2, r_st["rs"], p["backward_block.norm.weight"], dxh2)
    dz2 = dy2 * vm * silu_grad(z2)
    if delta is None:
        drin, grads["second_local.weight"], grads["second_local.bias"] = conv_backward(
            rin, p["second_local.weight"], dz2, dilation)
    else:
        drin, grads["second_local.weight"], grads["second_local.bias"] = physical_conv_backward(
            rin, p["second_local.weight"], parts2, samp2, dz2)
    dv = drin * vm
    # writer: synthesis + residual, then the block
    dmodal = ls * dv
    frame1 = p["forward_block.frame.weight"]
    grads["forward_block.layer_scale"] = np.sum(dv * (modal + ds * w_st["xh"]), axis=(0, 1))
    grads["forward_block.direct_scale"] = np.sum(dv * ls * w_st["xh"], axis=(0, 1))
    dframe_syn = np.einsum("btd,btj->dj", dmodal, s1)
    dxh1, dframe_drv, (grads["forward_block.raw_decay"], grads["forward_block.raw_frequency"]) = \
        _block_backward(y1, p, "forward_block", w_st, dm1, valid, extra_ds=dmodal @ frame1)
    grads["forward_block.frame.weight"] = dframe_syn + dframe_drv
    dxh1 = dxh1 + dv * ls * ds
    dy1_norm, grads["forward_block.norm.weight"] = rms_norm_backward(
        y1, w_st["rs"], p["forward_block.norm.weight"], dxh1)
    dy1 = dv + dy1_norm
    dz1 = dy1 * vm * silu_grad(z1)
    if delta is None:
        dproj, grads["stem.local.weight"], grads["stem.local.bias"] = conv_backward(
            proj, p["stem.local.weight"], dz1, dilation)
    else:
        dproj, grads["stem.local.weight"], grads["stem.local.bias"] = physical_conv_backward(
            proj, p["stem.local.weight"], parts1, samp1, dz1)
    grads["stem.projection.weight"] = np.einsum("btd,btc->dc", dproj, stem_in)
    return grads


__all__ = ["alphabet_backward", "moments_backward", "pole_backward", "radial_log_backward",
           "scan_backward"]
