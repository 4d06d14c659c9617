"""Generate ``tests/golden/refmerge_online.npz`` from the REFERENCE's own online track merge.

Run in a container that has the naver/blast3r checkout (not needed on the GPU box or by the
tests, which read the committed ``.npz``):

    B3R_REFERENCE=<path to blast3r checkout> python tests/golden/make_golden_merge.py

The online loop (``inference/pipeline.py:196-224``) grows its problem frame by frame with
``track_data = track_data | new_track_data``, ``ObservedTracks.__or__``
(``inference/tracks.py:96-117``).  This script takes a small seeded scene of the configs[3]
generator, forms for every frame q the reference's ``ObservedTracks`` of the tracks whose last
observation is in image q (the frame's new tracks, numbered from 0, over images 0..q), merges
them with the reference's own ``__or__`` and records each merged structure (observations per
image, track ids, and the keypoints, which identify the rows).  The tests check that
``blast3r_b200.synthetic.OnlineSequence`` builds the same problems.

``inference/tracks.py`` imports the track network, the retrieval processor and torch_scatter
at module level; the merge uses none of them, so they are replaced by empty stand-ins here.
"""
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from blast3r_b200.synthetic import make_scene   # noqa: E402

SCENE = dict(cfg=3, n_imgs=12, n_tracks=400, seed=301)


def reference_tracks_module(ref):
    sys.path.insert(0, os.path.join(ref, 'src'))
    sys.modules.setdefault('torch_scatter', types.ModuleType('torch_scatter'))
    models = types.ModuleType('blast3r.models')
    models.CausalTrack3R = object
    sys.modules['blast3r.models'] = models
    retr = types.ModuleType('blast3r.retrieval.processor')
    retr.IncrementalRetriever = object
    sys.modules['blast3r.retrieval.processor'] = retr
    import blast3r.inference.tracks as tracks
    return tracks


def frame_tracks(T, sc, q, last, img):
    """The reference ObservedTracks of the tracks last seen in image q, over images 0..q."""
    new = np.flatnonzero(last == q)                       # their ids in the scene, ascending
    renum = np.full(sc.n_tracks, -1)
    renum[new] = np.arange(len(new))
    sel = renum[sc.pids] >= 0
    # image-sorted, inside an image by (new) track id, as the reference lays tracks out
    order = np.lexsort((renum[sc.pids][sel], img[sel]))
    rows = np.flatnonzero(sel)[order]
    nppi = np.bincount(img[rows], minlength=q + 1)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))   # noqa: E731
    return T.ObservedTracks(q + 1, len(new), t(nppi), t(renum[sc.pids][rows].astype(np.int32)), t(sc.pix2d[rows]),
                            t(sc.pix2d_std[rows]), t(sc.pix2d_dep[rows]), 'log_multidepth')


def main():
    ref = os.environ.get('B3R_REFERENCE')
    if not ref:
        raise SystemExit('set B3R_REFERENCE to the blast3r checkout')
    T = reference_tracks_module(ref)
    sc = make_scene(SCENE['cfg'], n_imgs=SCENE['n_imgs'], n_tracks=SCENE['n_tracks'], seed=SCENE['seed'])
    img = np.repeat(np.arange(sc.n_imgs), np.diff(np.concatenate([[0], sc.infos[0]])))
    last = np.full(sc.n_tracks, -1)
    np.maximum.at(last, sc.pids, img)
    out = dict(scene_pids=sc.pids, scene_pix2d=sc.pix2d, scene_infos=sc.infos)
    track_data = None
    for q in range(sc.n_imgs):
        new = frame_tracks(T, sc, q, last, img)
        track_data = track_data | new                     # ObservedTracks.__or__ / __ror__
        out[f'f{q}_nppi'] = track_data.nppi.numpy()
        out[f'f{q}_pids'] = track_data.pids.numpy()
        out[f'f{q}_pix2d'] = track_data.pix2d.numpy()
        out[f'f{q}_n_tracks'] = np.array(track_data.n_tracks)
    path = os.path.join(HERE, 'refmerge_online.npz')
    np.savez_compressed(path, **out)
    print('wrote', path, 'frames', sc.n_imgs, 'final', int(track_data.n_tracks), 'tracks', len(track_data.pids), 'obs')


if __name__ == '__main__':
    main()
