"""Finetuning-job stages that exist only with adapter routing on (importing
this module registers them):

* ``indexing``  — build the job adapter's centroid from the job's dataset
  next to training (cached by dataset + encoder fingerprint);
* ``admission`` — after training: save the trained adapter as PEFT, then
  admit it to the pool (compared with the active set; the pool keeps serving
  throughout and a failed admission leaves it unchanged).

Reference: ``deltaserve-plugin/deltaserve/adapter_routing/stages.py:122-244``.
"""

from __future__ import annotations

import os

from ...engine.ft_job import Stage
from .indexing import store_centroid


class IndexingStage(Stage, key="indexing"):
    def prerequisites(self, listed):
        return tuple(k for k in ("init",) if k in listed)

    def begin(self, job, ctx) -> None:
        router = getattr(ctx, "router", None)
        if router is None:
            raise RuntimeError("adapter routing is not running")
        if not job.spec.data_path:
            raise RuntimeError("the job has no dataset to index")
        ijob, hit = router.index_job(job.spec.name, job.spec.data_path)
        job.data["indexing"] = (router, ijob, hit)

    def settled(self, job, ctx) -> bool:
        router, ijob, hit = job.data["indexing"]
        if hit is not None:
            job.data["centroid"] = hit
            return True
        if ijob.error:
            raise RuntimeError(ijob.error)
        if not ijob.done:
            return False
        c, r = ijob.indexer.centroid(), ijob.indexer.references()
        store_centroid(router.dir, job.spec.name, ijob.fp, c, r, router.enc_id,
                       router.cfg.encoder_query_prefix, router.cfg.encoder_max_tokens)
        job.data["centroid"] = (c, r)
        return True


class AdmissionStage(Stage, key="admission"):
    def prerequisites(self, listed):
        return tuple(k for k in listed if k not in (self.key, "ready"))   # after every other stage but ready

    def begin(self, job, ctx) -> None:
        router = getattr(ctx, "router", None)
        if router is None:
            raise RuntimeError("adapter routing is not running")
        path = job.spec.save_path or job.spec.adapter_path
        if "training" in job.spec.stages:
            root = job.spec.save_path or os.path.join(ctx.ftcfg.adapter_save_path or router.dir,
                                                      f"job-{job.spec.name}")
            path = ctx.save_adapter(root, save_id=f"job-{job.job_id}")
        if not path:
            raise RuntimeError("the job has no adapter to admit (no save_path / adapter_path)")
        c, r = job.data.get("centroid") or (None, None)
        job.report = router.pool.admit(job.spec.name, path, c, r, job=job.spec.name, load=True)
