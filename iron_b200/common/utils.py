"""Small helpers kept name-compatible with iron/common/utils.py."""


def float_to_name(v: float) -> str:
    """Filesystem-safe spelling of a float for operator names
    (iron/common/utils.py:22): repr() with '.'->'p', '-'->'n', '+' dropped."""
    return repr(v).replace(".", "p").replace("-", "n").replace("+", "")


DEVICE_NAME = "b200"
