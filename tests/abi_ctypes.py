"""Test-side view of the C ABI: the package's ctypes binding plus a parser
for the declarations in include/fa_b200.h."""
import os
import re

from flash_attention_sm75.capi import *  # noqa: F401,F403
from flash_attention_sm75.capi import LIB_PATH, SIGNATURES, fa_fwd, load, ptr, stream_ptr  # noqa: F401

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "fa_b200.h")


def header_functions():
    """Names of the functions declared in include/fa_b200.h."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*([a-z_][a-z0-9_]*)\s*\(",
                       text, flags=re.M)
    return sorted(set(names))
