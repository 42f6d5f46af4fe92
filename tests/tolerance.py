"""The BF16 tolerance of the north star, written once for every test:
max abs error <= 2e-2 and max abs error <= 1e-2 * max |reference| on the
compared hidden states."""

ABS_TOL = 2e-2
REL_TOL = 1e-2


def bf16_report(got, ref):
    g, r = got.detach().float().cpu(), ref.detach().float().cpu()
    err = (g - r).abs().max().item() if g.numel() else 0.0
    scale = r.abs().max().item() if r.numel() else 0.0
    return err, scale


def assert_bf16_close(got, ref, what=''):
    assert got.shape == ref.shape, f'{what}: shape {tuple(got.shape)} != {tuple(ref.shape)}'
    err, scale = bf16_report(got, ref)
    assert err <= ABS_TOL, f'{what}: max abs error {err:.3e} > {ABS_TOL}'
    assert err <= REL_TOL * max(scale, 1e-30) or err == 0.0, \
        f'{what}: max abs error {err:.3e} > {REL_TOL} x max|ref| ({scale:.3e})'
