"""``load`` of .npy / .npz / .csv files: ``TensorCompiler._load_data_file``
(tensorlang/compiler.py:68-162) and its call site (:1063-1104).

Same formats, selection rules, metadata and errors as the reference:

* ``.npy``: the array, as float32;
* ``.npz``: the named array if the program gives one (``KeyError`` naming
  the available arrays if it is missing), else the array called ``data``,
  else the first array in the file; ``columns`` and ``index`` arrays, when
  present, go into the metadata (byte strings decoded as UTF-8);
* ``.csv``: read with pandas; a first column called date, time, datetime,
  index or id (any case) becomes the metadata's index and is dropped; the
  rest must convert to float32 (``ValueError`` otherwise);
* any other suffix: ``ValueError`` listing the supported formats; a missing
  file: ``FileNotFoundError``.

Relative paths are taken from the current directory, as the reference does.
The loaded array must have the shape the type checker gave the tensor; the
reference prints a "Shape mismatch" message and fails the compile, here
``check_shape`` raises ``ValueError`` with the same facts.
"""
from __future__ import annotations

from pathlib import Path
from typing import Any, Dict, Optional, Tuple

import numpy as np

INDEX_COLUMNS = ("date", "time", "datetime", "index", "id")


def load_data_file(file_path: str, array_name: Optional[str] = None
                   ) -> Tuple[np.ndarray, Dict[str, Any]]:
    path = Path(file_path)
    if not path.is_absolute():
        path = Path.cwd() / path
    if not path.exists():
        raise FileNotFoundError(f"Data file not found: {file_path}")
    suffix = path.suffix.lower()
    meta: Dict[str, Any] = {"format": suffix[1:], "path": str(path)}
    if suffix == ".npy":
        data = np.load(path).astype(np.float32)
    elif suffix == ".npz":
        with np.load(path) as npz:
            names = list(npz.files)
            meta["available_arrays"] = names
            if array_name:
                if array_name not in names:
                    raise KeyError(f"Array '{array_name}' not found in {path.name}. "
                                   f"Available: {names}")
                pick = array_name
            else:
                pick = "data" if "data" in names else names[0]
            data = npz[pick].astype(np.float32)
            meta["array_name"] = pick
            if "columns" in names:
                meta["columns"] = npz["columns"].tolist()
            if "index" in names:
                idx = npz["index"]
                if idx.dtype.kind == "S":
                    meta["index"] = [x.decode("utf-8") if isinstance(x, bytes) else x for x in idx]
                else:
                    meta["index"] = idx.tolist()
    elif suffix == ".csv":
        import pandas as pd
        try:
            df = pd.read_csv(path)
        except Exception as e:
            raise ValueError(f"Failed to parse CSV file {path.name}: {e}")
        meta["rows"] = len(df)
        first = df.columns[0]
        if str(first).lower() in INDEX_COLUMNS:
            meta["index"] = df[first].tolist()
            df = df.drop(columns=[first])
        try:
            data = df.to_numpy().astype(np.float32)
        except ValueError as e:
            raise ValueError(f"CSV contains non-numeric data that cannot be converted to "
                             f"float32. Columns: {df.columns.tolist()}. Error: {e}")
        meta["columns"] = df.columns.tolist()
    else:
        raise ValueError(f"Unsupported file format: {suffix}. Supported formats: .npy, .npz, .csv")
    meta["shape"] = data.shape
    meta["dtype"] = "f32"
    return data, meta


def check_shape(name: str, file_path: str, data: np.ndarray, declared) -> np.ndarray:
    """The loaded array, if it has the declared shape (compiler.py:1074-1081)."""
    declared = tuple(int(d) for d in declared)
    if tuple(data.shape) != declared:
        raise ValueError(f"Shape mismatch: {file_path} (tensor {name})\n"
                         f"  File shape:     {tuple(data.shape)}\n"
                         f"  Declared shape: {declared}")
    return data
