"""The output specification's name tables for generated modules.

A module is valid only if every `THREE.X` it touches is an allowed member, every free identifier is an allowed
global, and it uses none of the forbidden names or properties. Downstream validators apply the same tables
(the reference keeps them in pipeline_service/modules/js_checker/validator/threeAllowlist.js and identifiers.js),
so these are an interface: a module this checker passes must pass theirs. The names are data; the rules that
use them are in `jscheck.static_analyze`, and the interpreter (`jsvm.make_three`) implements every allowed member.
"""
from __future__ import annotations

from typing import Dict, FrozenSet

# THREE.X members a module may use
THREE_ALLOWED: FrozenSet[str] = frozenset({
    # buffers and geometries
    "BufferGeometry", "BufferAttribute", "InterleavedBuffer", "InterleavedBufferAttribute",
    "Float32BufferAttribute", "Uint8BufferAttribute", "Uint16BufferAttribute", "Uint32BufferAttribute",
    "Int8BufferAttribute", "Int16BufferAttribute", "Int32BufferAttribute",
    "BoxGeometry", "SphereGeometry", "CylinderGeometry", "CapsuleGeometry", "ConeGeometry", "TorusGeometry",
    "TorusKnotGeometry", "PlaneGeometry", "CircleGeometry", "RingGeometry", "TetrahedronGeometry",
    "OctahedronGeometry", "DodecahedronGeometry", "IcosahedronGeometry", "PolyhedronGeometry", "ExtrudeGeometry",
    "LatheGeometry", "ShapeGeometry", "TubeGeometry", "EdgesGeometry", "WireframeGeometry",
    # materials and the one texture source
    "MeshStandardMaterial", "MeshPhysicalMaterial", "MeshBasicMaterial", "PointsMaterial", "LineBasicMaterial",
    "LineDashedMaterial", "DataTexture",
    # math
    "Vector2", "Vector3", "Vector4", "Matrix3", "Matrix4", "Quaternion", "Euler", "Box2", "Box3", "Sphere", "Plane",
    "Ray", "Line3", "Triangle", "Spherical", "Cylindrical", "Color", "MathUtils",
    # curves, paths and shapes
    "Curve", "CurvePath", "Shape", "Path", "CatmullRomCurve3", "CubicBezierCurve3", "LineCurve3",
    "QuadraticBezierCurve3", "EllipseCurve", "ArcCurve", "LineCurve", "SplineCurve", "QuadraticBezierCurve",
    "CubicBezierCurve",
    # scene objects
    "Object3D", "Group", "Mesh", "InstancedMesh", "Line", "LineSegments", "Points",
    # constants
    "SRGBColorSpace", "LinearSRGBColorSpace", "NoColorSpace", "FrontSide", "BackSide", "DoubleSide",
    "NormalBlending", "AdditiveBlending", "SubtractiveBlending", "MultiplyBlending", "NoBlending",
    "NearestFilter", "LinearFilter", "NearestMipmapNearestFilter", "LinearMipmapNearestFilter",
    "NearestMipmapLinearFilter", "LinearMipmapLinearFilter", "RepeatWrapping", "ClampToEdgeWrapping",
    "MirroredRepeatWrapping", "RGBAFormat", "RGBFormat", "RGFormat", "RedFormat", "LuminanceFormat",
    "UnsignedByteType", "HalfFloatType", "FloatType", "StaticDrawUsage", "DynamicDrawUsage", "StreamDrawUsage",
})

# members of allowed THREE.X that are themselves off limits
THREE_BLOCKED_SUBMEMBERS: Dict[str, FrozenSet[str]] = {"MathUtils": frozenset({"seededRandom", "generateUUID"})}

# real three.js members that are excluded on purpose (FORBIDDEN_THREE_API rather than UNKNOWN_THREE_API)
THREE_DISALLOWED_KNOWN: FrozenSet[str] = frozenset({
    # lights and shadows (the renderer lights the scene)
    "AmbientLight", "DirectionalLight", "PointLight", "SpotLight", "HemisphereLight", "RectAreaLight", "LightProbe",
    "AmbientLightProbe", "HemisphereLightProbe", "DirectionalLightShadow", "PointLightShadow", "SpotLightShadow",
    "LightShadow",
    # loaders (no network or files), core and add-on names
    "Loader", "LoadingManager", "FileLoader", "TextureLoader", "ImageLoader", "ImageBitmapLoader",
    "CubeTextureLoader", "DataTextureLoader", "BufferGeometryLoader", "MaterialLoader", "ObjectLoader",
    "FontLoader", "AudioLoader", "AnimationLoader", "CompressedTextureLoader", "GLTFLoader", "OBJLoader",
    "MTLLoader", "FBXLoader", "ColladaLoader", "STLLoader", "PLYLoader", "3MFLoader", "DRACOLoader", "KTX2Loader",
    "KTXLoader", "RGBELoader", "EXRLoader", "HDRCubeTextureLoader", "BasisTextureLoader", "TGALoader",
    "TIFFLoader", "SVGLoader", "USDZLoader", "VRMLLoader", "XYZLoader",
    # other materials
    "ShaderMaterial", "RawShaderMaterial", "MeshPhongMaterial", "MeshLambertMaterial", "MeshToonMaterial",
    "MeshNormalMaterial", "MeshMatcapMaterial", "MeshDepthMaterial", "MeshDistanceMaterial", "ShadowMaterial",
    "SpriteMaterial", "Material",
    # textures needing a DOM or compressed data
    "Texture", "CanvasTexture", "VideoTexture", "CompressedTexture", "CompressedArrayTexture",
    "CompressedCubeTexture", "CubeTexture", "Data3DTexture", "DataArrayTexture", "DepthTexture",
    "FramebufferTexture",
    # renderers, targets, cameras, scenes, fog (the validator owns the scene)
    "WebGLRenderer", "WebGL1Renderer", "WebGLRenderTarget", "WebGL3DRenderTarget", "WebGLArrayRenderTarget",
    "WebGLCubeRenderTarget", "WebGLMultipleRenderTargets", "Camera", "PerspectiveCamera", "OrthographicCamera",
    "ArrayCamera", "StereoCamera", "CubeCamera", "Scene", "Fog", "FogExp2",
    # animation
    "AnimationMixer", "AnimationAction", "AnimationClip", "AnimationObjectGroup", "AnimationUtils",
    "KeyframeTrack", "NumberKeyframeTrack", "VectorKeyframeTrack", "QuaternionKeyframeTrack",
    "ColorKeyframeTrack", "StringKeyframeTrack", "BooleanKeyframeTrack", "PropertyBinding", "PropertyMixer",
    # skinning, audio, sprites / LOD / batching
    "Bone", "Skeleton", "SkinnedMesh", "SkeletonHelper", "Audio", "PositionalAudio", "AudioAnalyser",
    "AudioContext", "AudioListener", "Sprite", "LOD", "BatchedMesh",
    # helpers and instrumentation
    "ArrowHelper", "AxesHelper", "BoxHelper", "Box3Helper", "CameraHelper", "GridHelper", "PolarGridHelper",
    "HemisphereLightHelper", "DirectionalLightHelper", "PointLightHelper", "SpotLightHelper", "PlaneHelper",
    "Raycaster", "Clock", "EventDispatcher", "Layers",
})

# free identifiers a module may reference (besides its own bindings)
ALLOWED_ROOT_IDENTIFIERS: FrozenSet[str] = frozenset({
    "Math", "Number", "String", "Array", "Object", "Symbol", "JSON", "Map", "Set", "Boolean", "Error", "TypeError",
    "RangeError", "Infinity", "NaN", "undefined", "parseInt", "parseFloat", "isFinite", "isNaN", "BigInt",
    "ArrayBuffer", "DataView", "Int8Array", "Uint8Array", "Uint8ClampedArray", "Int16Array", "Uint16Array",
    "Int32Array", "Uint32Array", "Float32Array", "Float64Array", "BigInt64Array", "BigUint64Array",
})

# names no binding or reference may use
FORBIDDEN_IDENTIFIERS: FrozenSet[str] = frozenset({
    "eval", "Function", "setTimeout", "setInterval", "setImmediate", "queueMicrotask", "fetch", "XMLHttpRequest",
    "WebSocket", "document", "window", "navigator", "localStorage", "sessionStorage", "indexedDB",
    "OffscreenCanvas", "HTMLCanvasElement", "crypto", "Date", "performance", "Proxy", "Reflect", "WeakRef",
    "FinalizationRegistry", "SharedArrayBuffer", "Atomics", "Worker", "process", "module", "global", "globalThis",
    "self", "require",
})

# roots on which computed member access (X[expr]) is rejected
COMPUTED_ACCESS_GATED: FrozenSet[str] = frozenset({"THREE", "Math", "Object", "Array", "Symbol"})

# property names no member access may use
FORBIDDEN_PROPERTY_NAMES: FrozenSet[str] = frozenset({
    "constructor", "__proto__", "__defineGetter__", "__defineSetter__", "__lookupGetter__", "__lookupSetter__",
})
