"""Scratch sizes of the weight-gradient plans, restated from minitensor_b200/csrc/mt_api.cu
(wgrad_plan and wgrad_tma_plan), so that tests can assert the exact byte counts the C ABI
reports or uses.

`sms` is the device's SM count as the library sees it: 148 on a B200, 0 where no device is
present (the host-only query then plans one split).
"""


def pick_bn(co):
    return 32 if co <= 32 else 64 if co <= 64 else 128 if co <= 128 else 256


def _splits(tiles, kb_total, sms):
    s = 1 if tiles >= sms else sms // tiles
    return max(1, min(s, kb_total))


def gather_bytes(N, C, Co, kh, kw, Ho, Wo, sms):
    """Split-K partials of the gather weight-gradient kernel: splits x C_out x (C kh kw) fp32."""
    M = C * kh * kw
    tiles = ((M + 127) // 128) * ((Co + pick_bn(Co) - 1) // pick_bn(Co))
    kb_total = N * ((Ho * Wo + 31) // 32)
    s = _splits(tiles, kb_total, sms)
    return (s * Co * M * 4 if s > 1 else 0), s


def tma_bytes(N, C, H, W, Co, kh, kw, Ho, Wo, sms, x3, x_in_place=False):
    """NHWC copy of x (channels padded to 4, rounded to 64 floats; none when x is already
    a channels-last copy, read in place) + split partials."""
    M = kh * kw * C
    bn = pick_bn(Co)
    # stage shape (runs of 32 pixels, rows): TF32 takes 2 rows per stage at C_out <= 64
    xcs, rs = (1, 1) if x3 else ((2, 2) if bn <= 64 else (2, 1))
    tiles_n = (Co + bn - 1) // bn
    tiles = ((M + 127) // 128) * tiles_n
    xblocks = (Wo + 32 * xcs - 1) // (32 * xcs)
    kb_total = N * ((Ho + rs - 1) // rs) * xblocks
    s = _splits(tiles, kb_total, sms)
    xt = 0 if x_in_place else N * H * W * ((C + 3) & ~3)
    xt = (xt + 63) & ~63
    return (xt + s * M * tiles_n * bn) * 4, s
