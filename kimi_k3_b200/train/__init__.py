"""Training services: optimizer, scheduler, engine, trainer loop, checkpoints, curriculum, diagnostics."""
