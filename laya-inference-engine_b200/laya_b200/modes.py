"""Mode selection with the b200 mode added (src/laya_blackwell/modes.py:4-19).

``create_engine(mode="b200", **options)`` builds a ``B200Engine``; the
reference's own modes ("balanced", "fast") are forwarded to the reference
package when it is installed.  Unknown modes fail before anything loads.
"""

MODES = ("balanced", "fast", "b200")


def create_engine(*, mode="balanced", **options):
    if mode == "b200":
        from .engine import B200Engine

        return B200Engine(**options)
    if mode in ("balanced", "fast"):
        try:
            from laya_blackwell.modes import create_engine as reference_create  # noqa: PLC0415
        except ImportError as exc:
            raise RuntimeError(f"mode {mode!r} needs the reference package laya_blackwell") from exc
        return reference_create(mode=mode, **options)
    raise ValueError("mode must be balanced, fast or b200")
