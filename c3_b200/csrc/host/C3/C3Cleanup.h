// Ordered shutdown of the C3 singletons (the reference's include/C3/C3Cleanup.h:34-40):
// hot-path manager -> backward capture -> engine (pending compiles, then cache) -> region
// registry -> kernel registry. Dropping the registries releases the CUDA kernel objects and
// the device memory they hold before static destruction.
#pragma once

#include "C3/C3BackwardCapture.h"
#include "C3/C3Engine.h"
#include "C3/C3HotPathManager.h"
#include "C3/RegionFusion.h"

namespace ct {
namespace c3 {

inline void shutdownAll() {
  C3HotPathManager::instance().shutdown();
  C3BackwardCapture::getInstance().waitForPendingCompiles();
  C3Engine::getInstance().shutdown();
  C3Engine::getInstance().clearCache();
  RegionFusionRegistry::getInstance().clear();
  C3KernelRegistry::getInstance().uninstallAll();
}

}  // namespace c3
}  // namespace ct
