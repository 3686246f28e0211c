"""Locations of the in-tree build products."""
import os

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_DIR = os.path.join(PKG, "lib")
CSRC = os.path.join(PKG, "csrc")


def main_lib() -> str:
    return os.path.join(LIB_DIR, "libstrasgpt.so")


def synth_lib() -> str:
    return os.path.join(LIB_DIR, "libstrasgpt_synth.so")


def include_dir() -> str:
    return os.path.join(ROOT, "include")
