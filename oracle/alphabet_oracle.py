"""CPU oracle for the ALPHABET forward path (numpy restatement).

TEST INFRASTRUCTURE ONLY.  This module is the parity checker: the `-m gpu`
tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import
it to compute the expected result of the CUDA path.  The product path in
``lnet_b200`` never imports, calls or falls back to it.

Every function restates one function of the reference ``lnet`` package and
cites it as ``path:line`` relative to the reference project root.  The
restatement is pinned against golden vectors produced by the reference itself
(``tests/golden/make_golden.py`` imports the reference on CPU and records its
inputs, parameters, stage outputs and logits; ``tests/test_oracle_golden.py``
checks this module against them).

Parameters are passed as a flat ``dict`` keyed by the reference
``state_dict`` names, except that each block's constrained frame is passed
materialised as ``"<block>.frame.weight"`` ([D, 2M]) instead of the
``parametrizations.weight.original``/``base`` pair.

Arithmetic precision is selectable: ``dtype=np.float32`` mirrors the
reference's fp32 tensors op for op, ``np.float64`` gives a higher-precision
reference of the same algorithm.
"""

from __future__ import annotations

import numpy as np

LAGS = (1, 2, 4)
DAMPING_MIN = 1.0e-3
DAMPING_MAX = 2.0
FP32_EPS = float(np.finfo(np.float32).eps)
FP32_TINY = float(np.finfo(np.float32).tiny)


def _f(a, dtype):
    return np.asarray(a, dtype=dtype)


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def silu(x):
    return x * sigmoid(x)


def damping_values(raw_decay, dtype=np.float64):
    """``_TightFrameBlock.damping_values`` (src/lnet/pac_tight_frame_models.py:487-491)."""
    raw = _f(raw_decay, dtype)
    return (DAMPING_MIN + (DAMPING_MAX - DAMPING_MIN) * sigmoid(raw)).astype(dtype)


def frequency_values(raw_frequency, dtype=np.float64):
    """``_TightFrameBlock.frequency_values`` (src/lnet/pac_tight_frame_models.py:458-459)."""
    return (np.pi * np.tanh(_f(raw_frequency, dtype))).astype(dtype)


def discrete_pole_real2d(damping, frequency, dt, threshold=1.0e-6, dtype=np.float64):
    """Exact zero-order hold of the complex pole ``p = -damping + i frequency``.

    Restates ``pole_transition_real2d`` and ``discrete_pole_real2d``
    (src/lnet/pac_real2d_math.py:20-29, :32-53): ``a = exp(p dt)`` and
    ``gamma = (a - 1) / p``, with ``gamma = dt`` when ``|p dt| < threshold``.
    Broadcasting follows numpy rules (``dt`` scalar or ``[B, T, 1]``).
    """
    d = _f(damping, dtype)
    w = _f(frequency, dtype)
    step = _f(dt, dtype)
    scaled = np.exp(-d * step)
    phase = w * step
    a_re = scaled * np.cos(phase)
    a_im = scaled * np.sin(phase)
    sh_re = a_re - 1.0
    sh_im = a_im
    p_re = -d
    p_im = w
    den = p_re * p_re + p_im * p_im
    g_re = (sh_re * p_re + sh_im * p_im) / den
    g_im = (sh_im * p_re - sh_re * p_im) / den
    small = np.sqrt((p_re * step) ** 2 + (p_im * step) ** 2) < threshold
    g_re = np.where(small, np.ones_like(g_re) * step, g_re)
    g_im = np.where(small, np.zeros_like(g_im), g_im)
    return (a_re.astype(dtype), a_im.astype(dtype), g_re.astype(dtype), g_im.astype(dtype))


def rms_norm(x, weight, dtype=np.float64):
    """``nn.RMSNorm(D)`` with ``eps=None`` -> fp32 machine epsilon
    (``_dtype_aligned_rms_norm``, src/lnet/pac_tight_frame_models.py:1850-1859)."""
    x = _f(x, dtype)
    ms = np.mean(x * x, axis=-1, keepdims=True)
    return (x / np.sqrt(ms + FP32_EPS) * _f(weight, dtype)).astype(dtype)


def same_length_dwconv(x, weight, bias, dilation=4):
    """Depthwise ``Conv1d(D, D, K, dilation, padding=dilation*(K-1)//2, groups=D)``
    applied on ``[B, T, D]`` (``_make_same_length_depthwise_conv1d``,
    src/lnet/pac_laplace_native_input.py:78-95)."""
    b, t, d = x.shape
    k = weight.shape[-1]
    w = weight.reshape(d, k)
    pad = dilation * (k - 1) // 2
    xp = np.zeros((b, t + 2 * pad, d), dtype=x.dtype)
    xp[:, pad : pad + t] = x
    out = np.zeros_like(x)
    for j in range(k):
        out += xp[:, j * dilation : j * dilation + t] * w[:, j]
    return out + bias.reshape(1, 1, d).astype(x.dtype)


def searchsorted_left(sorted_rows, queries):
    """Row-wise ``torch.searchsorted(right=False)``: first index with value >= query."""
    out = np.empty(queries.shape, dtype=np.int64)
    for b in range(sorted_rows.shape[0]):
        out[b] = np.searchsorted(sorted_rows[b], queries[b], side="left")
    return out


def lerp(a, b, w):
    """``torch.lerp`` on CPU: ``a + w (b - a)`` if ``|w| < 0.5`` else ``b - (b - a)(1 - w)``."""
    return np.where(np.abs(w) < 0.5, a + w * (b - a), b - (b - a) * (1.0 - w))


def timestamps_of(time_delta_b_t):
    """Row-wise cumulative sum of ``time_delta``.  The reference runs
    ``cumsum`` on CPU fp32 tensors, which accumulates in double and rounds
    every output to fp32."""
    acc = np.cumsum(time_delta_b_t.astype(np.float64), axis=1)
    return acc.astype(time_delta_b_t.dtype)


def physical_time_depthwise_conv(x, weight, bias, time_delta, valid_mask, dilation=4):
    """Depthwise kernel evaluated at fixed physical-time offsets on the
    piecewise-linear interpolant of ``x`` (``_physical_time_depthwise_conv``,
    src/lnet/alphabet_backbone.py:80-160).  ``time_delta`` is ``[B, T, 1]``,
    ``valid_mask`` ``[B, T, 1]`` or ``None``."""
    dtype = x.dtype
    b, t, d = x.shape
    k = weight.shape[-1]
    ts = timestamps_of(time_delta[..., 0])
    left = dilation * (k - 1) // 2
    offsets = (np.arange(k) * dilation - left).astype(dtype)
    queries = ts[:, :, None] + offsets[None, None, :]
    up_u = searchsorted_left(ts, queries.reshape(b, -1)).reshape(b, t, k)
    upper = np.minimum(up_u, t - 1)
    lower = np.clip(up_u - 1, 0, t - 1)
    bi = np.arange(b)[:, None, None]
    lt = ts[bi, lower]
    ut = ts[bi, upper]
    dur = ut - lt
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        interp = np.where(dur > 0, (queries - lt) / np.maximum(dur, FP32_TINY), 0.0)
    interp = np.clip(interp, 0.0, 1.0).astype(dtype)
    sampled = lerp(x[bi, lower], x[bi, upper], interp[..., None])
    in_bounds = (queries >= ts[:, :1, None]) & (queries <= ts[:, -1:, None])
    if valid_mask is not None:
        v = valid_mask[..., 0]
        lv = v[bi, lower]
        uv = v[bi, upper]
        eps8 = 8.0 * FP32_EPS
        support = np.where(interp <= eps8, lv, np.where(interp >= 1.0 - eps8, uv, lv * uv))
        in_bounds = in_bounds & (support > 0)
    sampled = sampled * in_bounds[..., None].astype(dtype)
    w = weight.reshape(d, k).astype(dtype)
    out = np.einsum("bnkd,dk->bnd", sampled, w)
    return (out + bias.reshape(1, 1, d)).astype(dtype)


def recurrence(a_re, a_im, u_re, u_im):
    """``s_t = a_t s_{t-1} + u_t`` from a zero state, real-2D complex form
    (``real2d_loop_recurrence``, src/lnet/pac_recurrence.py:191-212).
    ``a_*`` broadcast to ``[B, T, M]``."""
    bsz, t, m = u_re.shape
    a_re = np.broadcast_to(a_re, u_re.shape)
    a_im = np.broadcast_to(a_im, u_re.shape)
    s_re = np.empty_like(u_re)
    s_im = np.empty_like(u_im)
    cr = np.zeros((bsz, m), dtype=u_re.dtype)
    ci = np.zeros((bsz, m), dtype=u_re.dtype)
    for i in range(t):
        ar = a_re[:, i]
        ai = a_im[:, i]
        nr = ar * cr - ai * ci + u_re[:, i]
        ni = ai * cr + ar * ci + u_im[:, i]
        cr, ci = nr, ni
        s_re[:, i] = cr
        s_im[:, i] = ci
    return s_re, s_im


def modal_moments(s_re, s_im):
    """Unnormalised energy and lag-(1,2,4) autocorrelation means, order
    ``[E, C1r, C1i, C2r, C2i, C4r, C4i]`` (``_modal_moments`` with
    ``log_energy=False, normalize=False``, src/lnet/pac_tight_frame_models.py:1632-1657)."""
    out = [np.mean(s_re * s_re + s_im * s_im, axis=1)]
    for lag in LAGS:
        if s_re.shape[1] <= lag:
            z = np.zeros((s_re.shape[0], s_re.shape[2]), dtype=s_re.dtype)
            out += [z, z]
            continue
        cr, ci = s_re[:, lag:], s_im[:, lag:]
        pr, pi = s_re[:, :-lag], s_im[:, :-lag]
        out.append(np.mean(cr * pr + ci * pi, axis=1))
        out.append(np.mean(ci * pr - cr * pi, axis=1))
    return np.concatenate(out, axis=-1)


def masked_modal_moments(s_re, s_im, valid):
    """Valid-weighted moments with counts clamped at one
    (``_masked_modal_moments``, src/lnet/pac_tight_frame_models.py:1660-1702).
    ``valid`` is ``[B, T, 1]``."""
    mask = valid.astype(s_re.dtype)
    count = np.maximum(mask.sum(axis=1), 1.0)
    out = [((s_re * s_re + s_im * s_im) * mask).sum(axis=1) / count]
    for lag in LAGS:
        if s_re.shape[1] <= lag:
            z = np.zeros((s_re.shape[0], s_re.shape[2]), dtype=s_re.dtype)
            out += [z, z]
            continue
        w = mask[:, lag:] * mask[:, :-lag]
        wc = np.maximum(w.sum(axis=1), 1.0)
        cr, ci = s_re[:, lag:], s_im[:, lag:]
        pr, pi = s_re[:, :-lag], s_im[:, :-lag]
        out.append(((cr * pr + ci * pi) * w).sum(axis=1) / wc)
        out.append(((ci * pr - cr * pi) * w).sum(axis=1) / wc)
    return np.concatenate(out, axis=-1)


def interpolate_modal_state(s_re, s_im, ts, valid, queries):
    """Piecewise-linear state lookup at physical-time queries plus its support
    weight (``_interpolate_modal_state``, src/lnet/pac_tight_frame_models.py:1705-1752)."""
    b, t, _ = s_re.shape
    up_u = searchsorted_left(ts, queries)
    upper = np.minimum(up_u, t - 1)
    lower = np.clip(up_u - 1, 0, t - 1)
    bi = np.arange(b)[:, None]
    lt = ts[bi, lower]
    ut = ts[bi, upper]
    span = ut - lt
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        interp = np.where(span > 0, (queries - lt) / np.maximum(span, FP32_TINY), 0.0)
    interp = np.clip(interp, 0.0, 1.0).astype(s_re.dtype)
    pr = lerp(s_re[bi, lower], s_re[bi, upper], interp[..., None])
    pi = lerp(s_im[bi, lower], s_im[bi, upper], interp[..., None])
    v = valid[..., 0]
    lv = v[bi, lower]
    uv = v[bi, upper]
    eps8 = 8.0 * FP32_EPS
    support = np.where(interp <= eps8, lv, np.where(interp >= 1.0 - eps8, uv, lv * uv))
    in_bounds = (queries >= ts[:, :1]) & (queries <= ts[:, -1:])
    return pr, pi, support * in_bounds.astype(s_re.dtype)


def physical_time_modal_moments(s_re, s_im, time_delta, valid):
    """Duration-weighted energy and physical-time lag moments
    (``_physical_time_modal_moments``, src/lnet/pac_tight_frame_models.py:1755-1833).
    ``time_delta`` is ``[B, T, 1]``; ``valid`` ``[B, T, 1]`` or ``None``."""
    dtype = s_re.dtype
    delta = time_delta.astype(dtype)
    valid = np.ones_like(delta) if valid is None else valid.astype(dtype)
    ts = timestamps_of(delta[..., 0])
    dw = delta * valid
    dcount = dw.sum(axis=1)
    ecount = valid.sum(axis=1)
    use_d = dcount > 0
    ew = np.where(use_d[:, None, :], dw, valid)
    ec = np.maximum(np.where(use_d, dcount, ecount), 1.0)
    out = [((s_re * s_re + s_im * s_im) * ew).sum(axis=1) / ec]
    for lag in LAGS:
        q = (ts - float(lag)).astype(dtype)
        pr, pi, sup = interpolate_modal_state(s_re, s_im, ts, valid, q)
        pw = delta[..., 0] * valid[..., 0] * sup
        pc = np.maximum(pw.sum(axis=1, keepdims=True), 1.0)
        out.append(((s_re * pr + s_im * pi) * pw[..., None]).sum(axis=1) / pc)
        out.append(((s_im * pr - s_re * pi) * pw[..., None]).sum(axis=1) / pc)
    return np.concatenate(out, axis=-1)


def tight_frame_block(
    x,
    params,
    prefix,
    *,
    time_delta=None,
    event_mask=None,
    valid=None,
    moments_only=False,
    return_states=False,
):
    """One ``_TightFrameBlock.forward`` on the eager path used by ``Alphabet``
    (src/lnet/pac_tight_frame_models.py:717-1507; no local conv, tied frame,
    ``synthesis_scale == 1``, coupled residual scales, direction and moment
    direction "forward").  Returns ``moments`` or ``(stream, moments)``."""
    dtype = x.dtype
    norm_w = _f(params[prefix + ".norm.weight"], dtype)
    frame = _f(params[prefix + ".frame.weight"], dtype)  # [D, 2M]
    m = frame.shape[1] // 2
    normalized = rms_norm(x, norm_w, dtype)  # :812-813
    excitation = normalized @ frame  # :1038
    e_re, e_im = excitation[..., :m], excitation[..., m:]
    damping = damping_values(params[prefix + ".raw_decay"], dtype).reshape(1, 1, m)
    freq = frequency_values(params[prefix + ".raw_frequency"], dtype).reshape(1, 1, m)
    step = 1.0 if time_delta is None else time_delta.astype(dtype)
    a_re, a_im, g_re, g_im = discrete_pole_real2d(damping, freq, step, dtype=dtype)  # :1122-1141
    u_re = g_re * e_re - g_im * e_im  # :1145-1146
    u_im = g_re * e_im + g_im * e_re
    if event_mask is not None:  # :1147-1149
        u_re = event_mask.astype(dtype) * u_re
        u_im = event_mask.astype(dtype) * u_im
    s_re, s_im = recurrence(a_re, a_im, u_re.astype(dtype), u_im.astype(dtype))  # :1407-1414
    if time_delta is not None:  # :1421-1428
        moments = physical_time_modal_moments(s_re, s_im, time_delta.astype(dtype), valid)
    elif valid is not None:  # :1429-1435
        moments = masked_modal_moments(s_re, s_im, valid.astype(dtype))
    else:  # :1452-1457
        moments = modal_moments(s_re, s_im)
    if return_states:
        return s_re, s_im, moments
    if moments_only:
        return moments
    modal = np.concatenate([s_re, s_im], axis=-1) @ frame.T  # :1480, :1490
    ds = _f(params[prefix + ".direct_scale"], dtype)
    ls = _f(params[prefix + ".layer_scale"], dtype)
    out = x + ls * (modal + ds * normalized)  # :1503-1507
    return out.astype(dtype), moments


def radial_log_lag124(moments, modes):
    """``radial_log_lag124_moments`` (src/lnet/alphabet.py:29-46)."""
    dtype = moments.dtype
    out = [np.log1p(np.maximum(moments[..., :modes], 0.0))]
    for off in (modes, 3 * modes, 5 * modes):
        re = moments[..., off : off + modes]
        im = moments[..., off + modes : off + 2 * modes]
        r = np.sqrt(np.maximum(re * re + im * im, FP32_TINY))
        sc = np.log1p(r) / r
        out += [sc * re, sc * im]
    return np.concatenate(out, axis=-1).astype(dtype)


def prepare_metadata(x, time_delta, observation_mask, valid_mask, dtype):
    """Shape normalisation of request metadata
    (``_prepare_time_delta`` / ``_prepare_observation_mask`` / ``_prepare_mask``,
    src/lnet/alphabet_backbone.py:522-591).  Returns
    ``(delta [B,T,1], raw_obs [B,T,C|1], event_obs [B,T,1], valid [B,T,1])``."""

    def col(v):
        if v is None:
            return None
        v = _f(v, dtype)
        return v[..., None] if v.ndim == 2 else v

    delta = col(time_delta)
    raw = col(observation_mask)
    event = None
    if raw is not None:
        event = raw if raw.shape[-1] == 1 else raw.max(axis=-1, keepdims=True)  # :568
    valid = col(valid_mask)
    return delta, raw, event, valid


def edge_stem(x, params, delta, raw_obs, valid, dilation=4):
    """``AlphabetBackbone._edge_stem`` on the eager path
    (src/lnet/alphabet_backbone.py:593-676): mask raw values, project with
    ``P [D, C]``, same-length (or physical-time) depthwise conv, SiLU, mask."""
    dtype = x.dtype
    stem_in = x
    if raw_obs is not None:
        stem_in = stem_in * raw_obs
    if valid is not None:
        stem_in = stem_in * valid
    proj = stem_in @ _f(params["stem.projection.weight"], dtype).T
    w = _f(params["stem.local.weight"], dtype)
    bias = _f(params["stem.local.bias"], dtype)
    if delta is not None:
        local = physical_time_depthwise_conv(proj, w, bias, delta, valid, dilation)
    else:
        local = same_length_dwconv(proj, w, bias, dilation)
    first_local = silu(local).astype(dtype)
    if valid is not None:
        first_local = first_local * valid
    return first_local


def terminal_reader(first_stream, params, delta, valid, dilation=4):
    """``AlphabetBackbone._terminal_reader`` non-fused branch
    (src/lnet/alphabet_backbone.py:872-992): mask the writer stream, local
    conv (physical-time when ``delta`` is given), SiLU, mask, moments-only
    reader block (observation mask ``None``, :1170-1180 / alphabet.py:384-389)."""
    dtype = first_stream.dtype
    second = first_stream if valid is None else first_stream * valid
    w = _f(params["second_local.weight"], dtype)
    b = _f(params["second_local.bias"], dtype)
    if delta is not None:
        pre = physical_time_depthwise_conv(second, w, b, delta, valid, dilation)
    else:
        pre = same_length_dwconv(second, w, b, dilation)
    encoded = silu(pre).astype(dtype)
    if valid is not None:
        encoded = encoded * valid
    moments = tight_frame_block(
        encoded, params, "backward_block", time_delta=delta, event_mask=None, valid=valid,
        moments_only=True,
    )
    return encoded, moments


def alphabet_forward(
    x,
    params,
    *,
    time_delta=None,
    observation_mask=None,
    valid_mask=None,
    dtype=np.float64,
    return_stages=False,
):
    """``Alphabet.forward`` eager path (src/lnet/alphabet.py:350-416)."""
    x = _f(x, dtype)
    delta, raw_obs, event_obs, valid = prepare_metadata(
        x, time_delta, observation_mask, valid_mask, dtype
    )
    first_local = edge_stem(x, params, delta, raw_obs, valid)
    first_stream, first_moments = tight_frame_block(
        first_local, params, "forward_block", time_delta=delta, event_mask=event_obs, valid=valid
    )
    encoded, second_moments = terminal_reader(first_stream, params, delta, valid)
    m = _f(params["forward_block.frame.weight"], dtype).shape[1] // 2
    feats = np.concatenate(
        [radial_log_lag124(first_moments, m), radial_log_lag124(second_moments, m)], axis=-1
    )
    logits = feats @ _f(params["head.classifier.weight"], dtype).T + _f(
        params["head.classifier.bias"], dtype
    )
    if return_stages:
        return {
            "first_local": first_local,
            "first_stream": first_stream,
            "encoded": encoded,
            "writer_moments": first_moments,
            "reader_moments": second_moments,
            "logits": logits,
        }
    return logits


__all__ = [
    "alphabet_forward",
    "discrete_pole_real2d",
    "edge_stem",
    "masked_modal_moments",
    "modal_moments",
    "physical_time_depthwise_conv",
    "physical_time_modal_moments",
    "radial_log_lag124",
    "recurrence",
    "terminal_reader",
    "tight_frame_block",
]
