"""Weight files: the MTF format of aceflow/io/mtf.py, with loading to CUDA devices."""
from .mtf import MtfReader, load_model, load_mtf, save_model, save_mtf  # noqa: F401
