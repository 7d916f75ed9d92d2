def rel_err(out, ref):
    out = out.float()
    ref = ref.float()
    return float((out - ref).norm() / ref.norm().clamp(min=1e-12))


def assert_close(out, ref, tol=1e-2, what=""):
    e = rel_err(out, ref)
    assert e < tol, f"{what}: relative error {e:.3e} >= {tol}"
