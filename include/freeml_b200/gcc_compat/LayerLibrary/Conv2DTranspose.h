// GCC build compatibility for FreeML's Conv2DTranspose.h.
//
// LayerLibrary/Conv2DTranspose.h (lines 87, 98, 109 and 117) calls a member template of a
// dependent type without the `template` disambiguator
// (`blob->GetMatrix<Mat>(...)`), which MSVC accepts and GCC 13 rejects;
// Model.h reaches it through Loading/SaveLoader.h, so every GCC build of
// FreeML needs this.  Put this directory before the FreeML root on the
// include path: the header pre-includes what Conv2DTranspose.h depends on (all
// #pragma once), spells `GetMatrix` as `template GetMatrix` for the text of
// Conv2DTranspose.h only, and includes the real file from the next include directory.
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
#include_next <LayerLibrary/Conv2DTranspose.h>
#undef GetMatrix
