"""kvbm_b200.object: the G4 object tier's stores."""

from __future__ import annotations


def make_object_store(cfg, instance_id: str | None = None):
    """The store an ``ObjectConfig`` names: ``kind="fs"`` (directory ``root``) or ``kind="s3"``
    (``endpoint`` or AWS ``region``; credentials from the AWS_* environment variables)."""
    if cfg.kind == "fs":
        from .store import FsObjectStore

        if not cfg.root:
            raise ValueError("object store kind 'fs' needs a root directory")
        return FsObjectStore(cfg.root, cfg.bucket)
    if cfg.kind == "s3":
        from .s3 import S3Config, S3ObjectStore

        s3 = S3Config(endpoint_url=cfg.endpoint, bucket=cfg.bucket, region=cfg.region,
                      force_path_style=cfg.force_path_style if cfg.endpoint else False,
                      max_concurrent_requests=cfg.max_concurrent_requests)
        return S3ObjectStore(s3, instance_id=instance_id)
    raise ValueError(f"unknown object store kind {cfg.kind!r}")
