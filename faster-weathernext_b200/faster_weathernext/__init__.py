"""faster-weathernext on B200: the block-sparse masked flash attention of WeatherNext 2's mesh transformer.

    import faster_weathernext
    faster_weathernext.enable()          # select the B200 attention (options as the reference's)

The drop-in API of the reference (src/faster_weathernext/__init__.py:14-41): enable(force, **options)
updates `patch.OPTIONS` (a TypeError for an unknown option) and installs the patch; disable() uninstalls it;
options() returns the active Options. The attention itself is faster_weathernext.tiled_attn (C ABI in
libfwn_attn.so, include/fwn_attn.h).
"""

__version__ = "0.2.0+b200"


def enable(force: bool = False, **options):
  """Select the B200 attention path. Keyword options update faster_weathernext.patch.Options."""
  from faster_weathernext import patch
  for key in options:
    if not hasattr(patch.OPTIONS, key):
      raise TypeError(f"unknown option {key!r}; see faster_weathernext.patch.Options")
  for key, value in options.items():
    setattr(patch.OPTIONS, key, value)
  patch.warn_no_effect(options)
  patch.install(force=force)
  return patch.OPTIONS


def disable():
  from faster_weathernext import patch
  patch.uninstall()


def options():
  from faster_weathernext import patch
  return patch.OPTIONS
