// Build shim for compiling the unmodified FreeML headers with GCC.
//
// LayerLibrary/Conv2D.h (lines 83 and 96 upstream) calls a member template of a
// dependent type without the `template` disambiguator (`blob->GetMatrix<Mat>(...)`).
// MSVC accepts that; GCC 13 rejects it.  SaveLoader.h (pulled in by Model.h)
// includes this header, so the whole library fails to build on Linux.
//
// This shim sits before the FreeML root on the include path.  It first includes
// every header Conv2D.h depends on (they are #pragma once, so they are not read
// again), then defines `GetMatrix` as `template GetMatrix` for the text of
// Conv2D.h only, and pulls in the real header from the next include directory.
// The upstream file is compiled where it lies; nothing is copied or edited.
#pragma once
#include <LayerLibrary/Layer.h>
#include <LayerLibrary/Datablob.h>
#include <MatrixLibrary/MatrixBase.h>
#include <MatrixLibrary/MatrixInvalid.h>
#include <MatrixLibrary/MatrixBase_Functions.h>
#include <MatrixLibrary/GPU/DirectX11/MatrixDX11_Functions.h>
#include <ToolsLibrary/Tools.h>
#include <ActivationLibrary/Identity.h>
#define GetMatrix template GetMatrix
#include_next <LayerLibrary/Conv2D.h>
#undef GetMatrix
