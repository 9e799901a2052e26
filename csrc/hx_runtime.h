// Host-side runtime switches shared by every translation unit (plain C++).
#pragma once

// Process-wide switch for programmatic dependent launch (on by default).
inline bool& hx_pdl_enabled() {
  static bool on = true;
  return on;
}
