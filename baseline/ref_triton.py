"""The reference's own Triton GPU path, installed unmodified, as a GPU-side
oracle and as the GPU bar that the sm_100a kernels are timed against.

``python baseline/ref_triton.py`` (run where the reference checkout exists)
copies the reference's Triton operator packages, byte for byte, into
``baseline/_ref/`` (git-ignored; it travels with the working tree to the GPU
box) together with a SHA-256 manifest:

* ``ops/bev_pool/src/``  -> ``bev_pool_triton.bev_pool``  (bev_pool_triton.py:219-227)
* ``ops/voxel/src/``     -> ``voxelization_triton.hard_voxelize`` (:674-710),
  ``dynamic_voxelize`` (:428-463), ``scatter_points_triton.dynamic_point_to_voxel_forward``
  / ``_backward`` (:253-424)
* ``ops/spconv/src/``    -> ``spconv_triton.get_indice_pairs`` (:918-957), ``indice_conv``
  (:981-1007), ``indice_conv_backward`` (:1035-1061), ``indice_maxpool`` (:1064-1082)

The reference project has no installable package layout (``pip install``
fails on setuptools' flat-layout discovery), and importing its ``ops``
package pulls in compiled extensions that are not part of this path, so the
two ``src`` packages are loaded directly by ``load()`` under private names.
Nothing in ``bevfusion_triton_b200`` imports this module: only tests and the
benchmark do.
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / '_ref'
MANIFEST = REF_DIR / 'manifest.json'
PACKAGES = {'bev_pool_src': 'ops/bev_pool/src', 'voxel_src': 'ops/voxel/src', 'spconv_src': 'ops/spconv/src'}
SOURCE_ROOT = Path('/root/reference')


def _digest(p: Path) -> str:
    return hashlib.sha256(p.read_bytes()).hexdigest()


def install(source: Path = SOURCE_ROOT) -> dict:
    """Copy the reference's Triton packages unmodified into baseline/_ref."""
    files = {}
    for rel in PACKAGES.values():
        src = source / rel
        dst = REF_DIR / rel
        if dst.exists():
            shutil.rmtree(dst)
        dst.mkdir(parents=True)
        for f in sorted(src.glob('*.py')):
            shutil.copyfile(f, dst / f.name)
            files[f'{rel}/{f.name}'] = _digest(f)
    MANIFEST.write_text(json.dumps({'source': str(source), 'files': files}, indent=1, sort_keys=True))
    return files


def available() -> str | None:
    """None when the installed copy is present and intact, else why not."""
    if not MANIFEST.exists():
        return 'reference Triton path not installed (run baseline/ref_triton.py where the reference exists)'
    files = json.loads(MANIFEST.read_text())['files']
    for rel, want in files.items():
        p = REF_DIR / rel
        if not p.exists() or _digest(p) != want:
            return f'installed reference file {rel} is missing or modified'
    try:
        import triton  # noqa: F401
    except Exception as e:  # pragma: no cover
        return f'triton is not importable: {e}'
    return None


_mods: dict = {}


def _load_package(name: str, rel: str):
    pkg_dir = REF_DIR / rel
    spec = importlib.util.spec_from_file_location(name, pkg_dir / '__init__.py',
                                                  submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def load():
    """(bev_pool_triton, voxelization_triton, scatter_points_triton) modules of
    the installed reference.  Raises RuntimeError when it is unavailable."""
    if 'bev' in _mods:
        return _mods['bev'], _mods['vox'], _mods['scatter']
    why = available()
    if why:
        raise RuntimeError(why)
    _load_package('_bfbref_bev_pool_src', PACKAGES['bev_pool_src'])
    _load_package('_bfbref_voxel_src', PACKAGES['voxel_src'])
    _mods['bev'] = sys.modules['_bfbref_bev_pool_src.bev_pool_triton']
    _mods['vox'] = sys.modules['_bfbref_voxel_src.voxelization_triton']
    _mods['scatter'] = sys.modules['_bfbref_voxel_src.scatter_points_triton']
    return _mods['bev'], _mods['vox'], _mods['scatter']


def load_spconv():
    """The installed reference's ``spconv_triton`` module."""
    if 'spconv' in _mods:
        return _mods['spconv']
    why = available()
    if why:
        raise RuntimeError(why)
    if 'ops/spconv/src/spconv_triton.py' not in json.loads(MANIFEST.read_text())['files']:
        raise RuntimeError('the installed reference copy predates the spconv package: rerun baseline/ref_triton.py')
    _load_package('_bfbref_spconv_src', PACKAGES['spconv_src'])
    _mods['spconv'] = sys.modules['_bfbref_spconv_src.spconv_triton']
    return _mods['spconv']


if __name__ == '__main__':
    done = install()
    print(f'installed {len(done)} reference files into {REF_DIR}')
    print(available() or 'ok')
