import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "granite-speech-4.1-2b-nar-turbo_b200")
for _p in (ROOT, PKG, os.path.dirname(os.path.abspath(__file__))):
    if _p not in sys.path:
        sys.path.insert(0, _p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def pytest_sessionstart(session):
    # the library is built ahead of time; rebuild only if a source is newer than the .so
    from granite_conv_b200 import build
    if build.needs_build():
        build.build()


def pytest_terminal_summary(terminalreporter):
    """The bf16 parity checks of the session: the plain max-abs error beside the magnitude-relative gate."""
    import parity
    if not parity.RECORDS:
        return
    tr = terminalreporter
    lit = sum(1 for _, s in parity.RECORDS if s["max_abs"] <= parity.ATOL_BF16)
    tr.write_sep("-", f"bf16 parity: {len(parity.RECORDS)} comparisons, {lit} within a literal max-abs 2e-2")
    tr.write_line(f"{'check':60s} {'max|d|':>9s} {'max|ref|':>9s} {'<=2e-2':>6s} {'d/gate':>7s} {'rel-L2':>9s}")
    for what, s in parity.RECORDS:
        tr.write_line(f"{what[:60]:60s} {s['max_abs']:9.3e} {s['max_ref']:9.3g} "
                      f"{'yes' if s['max_abs'] <= parity.ATOL_BF16 else 'no':>6s} {s['worst_ratio']:7.3f} "
                      f"{s['rel_l2']:9.2e}")
