"""Model and device specs (TOML) and their loader."""
