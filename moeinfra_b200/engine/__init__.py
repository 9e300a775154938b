"""engine subsystem (B200 rebuild of the reference package of the same name)."""
